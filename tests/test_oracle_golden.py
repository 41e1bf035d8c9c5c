"""The CPU oracle against the reference's own known-answer tests
(vectors transcribed in tests/golden/reference_kat.json with citations)."""
import math

import numpy as np
import pytest

import oracle
import wgdec


def _want(v):
    return {"inf": math.inf, "-inf": -math.inf, "nan": math.nan}.get(v, v) if isinstance(v, str) else v


def test_f16_to_f32_known_answers(kat):
    # internal/gguf/gguf_test.go:155-186
    for case in kat["f16_to_f32"]:
        got = oracle.f16_to_f32(case["h"])
        want = _want(case["want"])
        if isinstance(want, float) and math.isnan(want):
            assert math.isnan(got), case
        else:
            assert got == want, case
            assert math.copysign(1, got) == math.copysign(1, want), case


def test_f16_to_f32_exhaustive_against_ieee():
    hs = np.arange(65536, dtype=np.uint16)
    ref = hs.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(h)) for h in hs], dtype=np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(ref))


@pytest.mark.parametrize("idx", range(5))
def test_dequant_known_answers(kat, idx):
    # internal/gguf/gguf_test.go:190-309
    case = kat["dequant"][idx]
    out = oracle.dequant(case["qtype"], bytes(case["block"]), case["n"])
    for k, v in case["want"].items():
        assert out[int(k)] == v, (case["src"], k, out[int(k)], v)


@pytest.mark.parametrize("idx", range(6))
def test_quant_roundtrip_bounds(kat, idx):
    # internal/gguf/quant_test.go:11-85
    case = kat["quant_roundtrip"][idx]
    x = (np.arange(32, dtype=np.float32) / np.float32(31) * np.float32(2) - np.float32(1)).astype(np.float32)
    enc = wgdec.quantize(case["qtype"], x)
    dec = oracle.dequant(case["qtype"], enc, 32)
    assert np.max(np.abs(dec - x)) <= case["max_err"], case


def test_f16_conversion_roundtrip(kat):
    # internal/gguf/quant_test.go:88-127
    for case in kat["f16_conversion"]:
        h = oracle.f32_to_f16(case["f32"])
        got = oracle.f16_to_f32(h)
        tol = case["max_err"] or max(abs(case["f32"]) * 1e-3, 1e-6)
        assert abs(case["f32"] - got) <= tol, case


def test_f32_to_f16_matches_generator_and_ieee_off_ties():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10 ** rng.uniform(-8, 4, 20000),
                         np.array([0, -0.0, 65504, 65520, 1e-8, 6e-5, 6.1e-5, np.inf, -np.inf], np.float32)])
    g = wgdec.gen()
    for x in xs.astype(np.float32):
        a = oracle.f32_to_f16(float(x))
        assert a == g.wg_gen_f32_to_f16(float(x))
        # away from round-half ties and the f16 subnormal range, IEEE round-to-nearest agrees
        bits = int(np.float32(x).view(np.uint32))
        exp16 = ((bits >> 23) & 0xFF) - 127 + 15
        if 0 < exp16 < 31 and (bits & 0x1FFF) != 0x1000:
            assert a == int(np.float16(x).view(np.uint16)), x


@pytest.mark.parametrize("case_idx", range(4))
def test_gelu_known_values(kat, case_idx):
    # internal/ml/ops_test.go:223-240
    c = kat["gelu"][case_idx]
    assert abs(oracle.gelu(np.array([c["x"]], np.float32))[0] - c["want"]) <= c["tol"]


def test_layernorm_known_values(kat):
    # internal/ml/ops_test.go:243-286
    c = kat["layernorm"][0]
    got = oracle.layernorm(np.array([c["x"]], np.float32), np.array(c["w"], np.float32), np.array(c["b"], np.float32))
    assert np.max(np.abs(got[0] - np.array(c["want"]))) <= c["tol"]
    c = kat["layernorm"][1]
    got = oracle.layernorm(np.array([c["x"]], np.float32), np.array(c["w"], np.float32), np.array(c["b"], np.float32))
    assert abs(float(got.mean())) <= c["mean_tol"]
    assert abs(float(((got - got.mean()) ** 2).mean()) - 1) <= c["var_tol"]


def test_attention_causal_known_values(kat):
    # internal/ml/ops_test.go:349-438
    c = kat["attention"]
    q = np.array(c["q"], np.float32).reshape(c["shape"])
    out = oracle.attention(q, q, q, causal=True)
    assert np.allclose(out[0, 0], c["causal_out0"], atol=1e-5)
    e05 = math.exp(0.5)
    assert abs(out[0, 1, 0] - 1 / (1 + e05)) <= c["tol"]
    assert abs(out[0, 1, 1] - e05 / (1 + e05)) <= c["tol"]


def test_attention_fast_softmax_close_to_exact(kat):
    # internal/ml/attention_test.go:9-60 (seeded uniform [-1, 1) inputs)
    rng = np.random.default_rng(7)
    q, k, v = [(rng.random((4, 32, 64), dtype=np.float32) - 0.5) * 2 for _ in range(3)]
    fast = oracle.attention(q, k, v, causal=False)
    s = np.einsum("hqd,hkd->hqk", q.astype(np.float64), k.astype(np.float64)) / 8.0
    p = np.exp(s - s.max(-1, keepdims=True))
    exact = np.einsum("hqk,hkd->hqd", p / p.sum(-1, keepdims=True), v.astype(np.float64))
    assert np.max(np.abs(fast - exact)) <= kat["attention"]["fast_vs_exact"]["max_abs"]


def test_fast_exp_bounds():
    xs = np.linspace(-19.9, 0, 4001, dtype=np.float32)
    got = np.array([oracle.fast_exp(float(x)) for x in xs])
    assert np.max(np.abs(got / np.exp(xs.astype(np.float64)) - 1)) < 2e-3  # 4th-order Taylor on [0, ln2)
    assert oracle.fast_exp(-20.0) == 0.0 and oracle.fast_exp(0.0) == 1.0


def test_dot_q8_known_case(kat):
    # internal/ml/matmul_q8_test.go:95-114
    i = np.arange(64)
    f = (i % 7 - 3).astype(np.float32)
    g = ((i * 3) % 11 - 5).astype(np.float32)
    q = wgdec.quantize("Q8_0", g)
    assert abs(oracle.dot_row("Q8_0", q, f) - float(np.dot(f, g))) <= kat["dot_q8"]["tol"]


def test_matmul_q8_known_case(kat):
    # internal/ml/matmul_q8_test.go:116-149
    c = kat["matmul_q8"]
    a = (((np.arange(c["m"] * c["k"]) % 13) - 6) * 0.1).astype(np.float32).reshape(c["m"], c["k"])
    b = (((np.arange(c["n"] * c["k"]) % 9) - 4) * 0.2).astype(np.float32).reshape(c["n"], c["k"])
    got = oracle.matmul("Q8_0", wgdec.quantize_matrix("Q8_0", b), c["n"], c["k"], a)
    assert np.max(np.abs(got - a @ b.T)) <= c["tol"]


@pytest.mark.parametrize("qt", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"])
def test_matmul_all_types_known_case(kat, qt):
    # internal/ml/matmul_q8_test.go:151-207
    c = kat["matmul_all"]
    a = (((np.arange(c["m"] * c["k"]) % 17) - 8) * 0.07).astype(np.float32).reshape(c["m"], c["k"])
    b = (((np.arange(c["n"] * c["k"]) % 11) - 5) * 0.11).astype(np.float32).reshape(c["n"], c["k"])
    got = oracle.matmul(qt, wgdec.quantize_matrix(qt, b), c["n"], c["k"], a)
    assert np.max(np.abs(got - a @ b.T)) <= c["tols"][qt]


@pytest.mark.parametrize("qt", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"])
def test_dot_equals_dequant_dot(qt):
    """The per-type dot kernels agree with dequant-then-dot (float32 rounding level)."""
    rng = np.random.default_rng(3)
    w = rng.standard_normal((7, 96)).astype(np.float32) * 0.02
    a = rng.standard_normal((3, 96)).astype(np.float32)
    raw = wgdec.quantize_matrix(qt, w)
    deq = oracle.dequant(qt, raw, w.size).reshape(w.shape)
    got = oracle.matmul(qt, raw, 7, 96, a)
    assert np.allclose(got, a.astype(np.float64) @ deq.T.astype(np.float64), atol=1e-5, rtol=1e-5)
