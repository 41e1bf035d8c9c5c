"""wg_model_matmul_noalloc: the tcgen05 GEMM on a model's uploaded weights
with caller-owned device buffers and the library's fixed split-K scratch
(no device allocation in the call). Its results must match wg_matmul_test,
which runs the same kernel with an allocated workspace, on the same
quantised matrix and the same f16 activations, on two calls in a row.
This file sorts last so the scratch is also exercised after every other
GPU test of the session."""
import ctypes

import numpy as np
import pytest

import wgdec

pytestmark = pytest.mark.gpu

ERR_INVALID = 1  # WG_ERR_INVALID
# same kernel and K split on both sides; the tolerance only absorbs a
# different split choice (fp32 partial sums in another grouping)
ATOL, RTOL = 1e-3, 1e-4


def _last_error():
    buf = ctypes.create_string_buffer(512)
    wgdec.lib().wg_last_error(buf, len(buf))
    return buf.value.decode()


def _raw(mat):
    """Raw GGUF bytes of a model-descriptor matrix (Q8_0: 34 bytes per 32 values)."""
    assert mat.qtype == wgdec.QTYPES["Q8_0"]
    return ctypes.string_at(mat.data, mat.rows * (mat.cols // 32) * 34)


def _weights(model, layer, which):
    """(raw bytes, rows, cols) of matrix `which` of the device model, as uploaded
    (self-attention q, k, v stacked in that order)."""
    ly = wgdec._desc_ptr(model).contents.layers[layer]
    if which == 0:
        mats = [ly.self_q, ly.self_k, ly.self_v]
        return b"".join(_raw(m) for m in mats), sum(m.rows for m in mats), ly.self_q.cols
    m = [None, ly.self_o, ly.cross_q, ly.cross_o, ly.mlp0, ly.mlp2][which]
    return _raw(m), m.rows, m.cols


@pytest.fixture(scope="module")
def setup():
    torch = pytest.importorskip("torch")
    model = wgdec.SyntheticModel(51864, 256, 4, 2, 448, "Q8_0", seed=29)
    dec = wgdec.WhisperDecoder(model, devices=[0])
    yield torch, model, dec
    dec.close()
    model.close()


def _noalloc(torch, dec, layer, which, x16, n_out, wait=1):
    rows = x16.shape[0]
    out = torch.full((rows, n_out), float("nan"), dtype=torch.float32, device="cuda:0")
    rc = wgdec.lib().wg_model_matmul_noalloc(dec.h, 0, layer, which, x16.data_ptr(), x16.shape[1], rows,
                                             out.data_ptr(), n_out, None, wait)
    return rc, out


@pytest.mark.parametrize("which", range(6))
def test_matches_the_allocating_entry_point_twice(setup, which):
    torch, model, dec = setup
    raw, n, k = _weights(model, 1, which)
    rng = np.random.default_rng(100 + which)
    x = rng.standard_normal((40, k)).astype(np.float16)  # 40 rows: K split over a cluster
    ref = wgdec.matmul("Q8_0", raw, n, k, x.astype(np.float32), path=3)
    x16 = torch.from_numpy(x).to("cuda:0")
    for _ in range(2):
        rc, out = _noalloc(torch, dec, 1, which, x16, n)
        assert rc == 0, _last_error()
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_rejects_shapes_beyond_the_scratch(setup):
    """mlp.0 (1024 x 256) at 2048 rows: 64 output tiles, so a K split of 2 or
    more would need 64 x ks x 256 x 128 floats, beyond the 2 Mi of the
    scratch; the call must refuse it, or (where occupancy leaves the K
    unsplit and no scratch is needed) give the allocating entry point's result."""
    torch, model, dec = setup
    raw, n, k = _weights(model, 0, 4)
    x = np.random.default_rng(7).standard_normal((2048, k)).astype(np.float16)
    x16 = torch.from_numpy(x).to("cuda:0")
    rc, out = _noalloc(torch, dec, 0, 4, x16, n)
    if rc == ERR_INVALID:
        msg = _last_error()
        assert "wg_model_matmul_noalloc" in msg and "scratch" in msg
    else:
        assert rc == 0, _last_error()
        ref = wgdec.matmul("Q8_0", raw, n, k, x.astype(np.float32), path=3)
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_rejects_bad_layouts(setup):
    torch, model, dec = setup
    x16 = torch.zeros((40, 260), dtype=torch.float16, device="cuda:0")  # ldx % 8 != 0
    rc, _ = _noalloc(torch, dec, 0, 1, x16, 256)
    assert rc == ERR_INVALID
    x16 = torch.zeros((40, 256), dtype=torch.float16, device="cuda:0")
    rc, _ = _noalloc(torch, dec, 2, 1, x16, 256)  # layer out of range
    assert rc == ERR_INVALID
