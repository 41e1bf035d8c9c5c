"""Kernel-level parity on the GPU through the C ABI: bit-exact dequantisation
(the reference's dequant known answers + random blocks) and the fused
dequant GEMV/GEMM against the oracle."""
import numpy as np
import pytest

import oracle
import wgdec

pytestmark = pytest.mark.gpu
QT = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"]
BLOCK = {"Q4_0": 18, "Q4_1": 20, "Q5_0": 22, "Q5_1": 24, "Q8_0": 34}
SCALES = {"Q4_0": [0], "Q4_1": [0, 2], "Q5_0": [0], "Q5_1": [0, 2], "Q8_0": [0]}


@pytest.mark.parametrize("idx", range(5))
def test_dequant_known_answers_gpu(kat, idx):
    # internal/gguf/gguf_test.go:190-309, through the device layout
    case = kat["dequant"][idx]
    out = wgdec.dequant(case["qtype"], bytes(case["block"]), case["n"])
    for k, v in case["want"].items():
        assert out[int(k)] == v, (case["src"], k)


def random_blocks(qt, nblocks, seed):
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(nblocks, BLOCK[qt]), dtype=np.uint8)
    # finite f16 scales / mins (normal and subnormal magnitudes)
    for off in SCALES[qt]:
        h = (rng.standard_normal(nblocks) * 10.0 ** rng.uniform(-6, 1, nblocks)).astype(np.float16)
        raw[:, off:off + 2] = h.view(np.uint8).reshape(nblocks, 2)
    return raw.tobytes()


@pytest.mark.parametrize("qt", QT)
@pytest.mark.parametrize("n", [32, 32 * 37, 32 * 1000 - 5])
def test_dequant_bit_exact_random(qt, n):
    raw = random_blocks(qt, (n + 31) // 32, seed=n)
    gpu = wgdec.dequant(qt, raw, n)
    ref = oracle.dequant(qt, raw, n)
    assert np.array_equal(gpu.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qt", ["F32", "F16"])
def test_dequant_dense(qt):
    x = np.random.default_rng(5).standard_normal(1000).astype(np.float32)
    raw = x.tobytes() if qt == "F32" else x.astype(np.float16).tobytes()
    assert np.array_equal(wgdec.dequant(qt, raw, 1000), oracle.dequant(qt, raw, 1000))


def _matmul_case(qt, R, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    a = rng.standard_normal((R, cols)).astype(np.float32)
    raw = wgdec.quantize_matrix(qt, w)
    return raw, a, oracle.matmul(qt, raw, rows, cols, a)


# Tolerance of the fused dequant kernels (f16 tensor-core operands, fp32
# accumulation) against the oracle's fp32 dot products: the decoder's
# relative gate, max |err| <= 1e-3 * max |reference|. (x enters these unit
# calls rounded to f16 once; the weights enter as f16 high + low parts on
# the small-batch and tcgen05 paths.)
def _close(gpu, ref):
    return np.max(np.abs(gpu - ref)) <= 1e-3 * float(np.max(np.abs(ref)))


@pytest.mark.parametrize("qt", QT)
@pytest.mark.parametrize("R,path", [(1, 1), (5, 1), (8, 1), (13, 1), (16, 1), (16, 2), (40, 2), (130, 2), (5, 2),
                                    (1, 4), (5, 4), (16, 4)])
def test_matmul_vs_oracle(qt, R, path):
    raw, a, ref = _matmul_case(qt, R, 200, 256, seed=R * 7 + path)
    gpu = wgdec.matmul(qt, raw, 200, 256, a, path=path)
    assert _close(gpu, ref), float(np.max(np.abs(gpu - ref)))


@pytest.mark.parametrize("qt", QT)
@pytest.mark.parametrize("R", [17, 40, 130, 320])
def test_matmul_tcgen05_vs_oracle(qt, R):
    """The tcgen05 path (TMA-fed, TMEM accumulators) on partial weight and row tiles."""
    raw, a, ref = _matmul_case(qt, R, 200, 256, seed=R * 13)
    gpu = wgdec.matmul(qt, raw, 200, 256, a, path=3)
    assert _close(gpu, ref), float(np.max(np.abs(gpu - ref)))


@pytest.mark.parametrize("R,rows,K", [(320, 1280, 1280), (600, 384, 5120), (40, 5120, 1280), (1500, 256, 384)])
def test_matmul_tcgen05_model_shapes(R, rows, K):
    raw, a, ref = _matmul_case("Q8_0", R, rows, K, seed=R + K)
    gpu = wgdec.matmul("Q8_0", raw, rows, K, a, path=3)
    assert _close(gpu, ref), float(np.max(np.abs(gpu - ref)))


@pytest.mark.parametrize("qt", ["Q8_0", "Q5_1"])
@pytest.mark.parametrize("R,rows,K", [(5, 1280, 5120), (1, 3840, 1280), (16, 5120, 1280), (5, 1300, 1280),
                                      (3, 2000, 768), (24, 1280, 1280), (40, 3840, 1280), (40, 1280, 5120),
                                      (48, 5120, 1280), (33, 1300, 768)])
def test_matmul_small_batch_model_shapes(qt, R, rows, K):
    """The small-batch GEMV (path 1: a 128-row weight group per CTA, K ranges
    summed across a thread-block cluster) at decoder shapes up to 48 rows,
    with partial weight groups and K split into up to 16 ranges."""
    raw, a, ref = _matmul_case(qt, R, rows, K, seed=R + rows + K)
    gpu = wgdec.matmul(qt, raw, rows, K, a, path=1)
    assert _close(gpu, ref), float(np.max(np.abs(gpu - ref)))


@pytest.mark.parametrize("qt", QT)
def test_matmul_reference_tolerances(kat, qt):
    # internal/ml/matmul_q8_test.go:151-207 on the device (K=64 -> two quant blocks)
    c = kat["matmul_all"]
    a = (((np.arange(c["m"] * c["k"]) % 17) - 8) * 0.07).astype(np.float32).reshape(c["m"], c["k"])
    b = (((np.arange(c["n"] * c["k"]) % 11) - 5) * 0.11).astype(np.float32).reshape(c["n"], c["k"])
    got = wgdec.matmul(qt, wgdec.quantize_matrix(qt, b), c["n"], c["k"], a)
    assert np.max(np.abs(got - a @ b.T)) <= c["tols"][qt]


@pytest.mark.parametrize("qt", ["F32", "F16"])
def test_matmul_dense(qt):
    rng = np.random.default_rng(11)
    w = rng.standard_normal((37, 20)).astype(np.float32)
    a = rng.standard_normal((3, 20)).astype(np.float32)
    raw = w.tobytes() if qt == "F32" else w.astype(np.float16).tobytes()
    ref = oracle.matmul(qt, raw, 37, 20, a)
    assert _close(wgdec.matmul(qt, raw, 37, 20, a), ref)


@pytest.mark.parametrize("K", [384, 1280, 5120])
def test_matmul_model_shapes(K):
    raw, a, ref = _matmul_case("Q8_0", 5, 1280, K, seed=K)
    assert _close(wgdec.matmul("Q8_0", raw, 1280, K, a), ref)
