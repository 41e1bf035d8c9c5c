"""Decoder-level parity on the GPU through the C ABI against the CPU oracle.

Tolerances (the north-star gate): teacher-forced logits within max-abs 2e-2
and rel 1e-3 on every step, rel read as max|gpu - ref| / max|ref| (fp32
accumulation; weights and LayerNorm outputs enter the tensor-core products
as f16 high + low parts, f16 KV caches). Greedy tokens must be identical at every step whose oracle top-2
margin exceeds 2e-2; comparison stops at the first step under the margin."""
import threading

import numpy as np
import pytest

import oracle
import wgdec

pytestmark = pytest.mark.gpu
ATOL, RTOL, MARGIN = 2e-2, 1e-3, 2e-2
PROMPT = [50258, 50259, 50357, 50363]


@pytest.fixture(scope="module")
def tiny():
    m = wgdec.SyntheticModel(51864, 384, 6, 4, 448, "Q8_0", seed=11)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


def assert_logits_close(gpu, ref):
    """Per step: max-abs <= ATOL and max-abs <= RTOL * max|ref|."""
    gpu, ref = np.atleast_2d(gpu), np.atleast_2d(ref)
    for s in range(ref.shape[0]):
        err = float(np.max(np.abs(gpu[s] - ref[s])))
        assert err <= ATOL, "step %d: max abs err %.3g" % (s, err)
        assert err <= RTOL * float(np.max(np.abs(ref[s]))), "step %d: max abs err %.3g > %g * max|ref|" % (
            s, err, RTOL)


@pytest.mark.parametrize("mode", [wgdec.MODE_REF_COMPAT, wgdec.MODE_CORRECT])
def test_teacher_forced_tiny(tiny, mode):
    m, dec = tiny
    enc = m.encoder_output(0)
    forced = np.random.default_rng(mode).integers(0, 50257, size=8)
    ref = oracle.teacher_forced(m, enc, PROMPT, forced, mode, m.n_vocab)
    gpu = dec.teacher_forced_logits(enc, PROMPT, forced, mode)[:, 0, :]
    assert_logits_close(gpu, ref)


@pytest.mark.parametrize("xattn", ["stream", "cluster"])
def test_teacher_forced_cross_attention_kernels(tiny, xattn, monkeypatch):
    """Both cross-attention kernels (cluster split / streaming two-pass) on a 2-utterance batch."""
    m, dec = tiny
    monkeypatch.setenv("WG_XATTN", xattn)
    encs = [m.encoder_output(u) for u in (5, 6)]
    forced = np.random.default_rng(9).integers(0, 50257, size=(2, 4))
    gpu = dec.teacher_forced_logits(encs, PROMPT, forced, wgdec.MODE_CORRECT)
    for u in range(2):
        ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], wgdec.MODE_CORRECT, m.n_vocab)
        assert_logits_close(gpu[:, u, :], ref)


def margins_along(m, enc, toks, params, mode):
    """Oracle top-2 margins of the penalised logits along a token sequence."""
    P = len(params.prompt)
    forced = toks[P:]
    lg = oracle.teacher_forced(m, enc, params.prompt, forced, mode, m.n_vocab)
    out = []
    for s in range(len(forced)):
        pl = oracle.apply_penalty(lg[s], toks[:P + s])
        top2 = np.sort(pl)[-2:]
        out.append(float(top2[1] - top2[0]))
    return out


def assert_tokens_match_until_tie(m, enc, gpu_toks, ref_toks, params, mode):
    P = len(params.prompt)
    margins = margins_along(m, enc, ref_toks, params, mode)
    n = 0
    for s, mg in enumerate(margins):
        if mg <= MARGIN:
            break
        assert gpu_toks[P + s] == ref_toks[P + s], "step %d (margin %.3g)" % (s, mg)
        n += 1
    return n


@pytest.mark.parametrize("mode", [wgdec.MODE_REF_COMPAT, wgdec.MODE_CORRECT])
@pytest.mark.parametrize("beam", [1, 5])
def test_decode_tokens_tiny(tiny, mode, beam):
    m, dec = tiny
    encs = [m.encoder_output(u) for u in range(3)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=beam, max_tokens=16, mode=mode)
    gt, gl, _ = dec.decode_tokens(encs, params)
    rt, rl, _ = oracle.decode(m, encs, params, 448, threads=4)
    for u in range(3):
        assert gt[u, :4].tolist() == PROMPT
        assert_tokens_match_until_tie(m, encs[u], gt[u, :gl[u]], rt[u, :rl[u]], params, mode)


def reference_test_model(kat):
    """The hand-made decoder of internal/model/decoder_test.go:21-86 (F32, all weights 0.01)."""
    c = kat["decoder_tests"]
    V, d, H, ctx = c["n_vocab"], c["d"], c["heads"], c["ctx"]
    small = lambda *s: np.full(s, 0.01, np.float32)
    mat = lambda r, k: ("F32", r, k, small(r, k))
    ones, zeros = np.ones(d, np.float32), np.zeros(d, np.float32)
    layer = dict(self_ln_w=ones, self_ln_b=zeros, self_q=mat(d, d), self_q_b=zeros, self_k=mat(d, d),
                 self_v=mat(d, d), self_v_b=zeros, self_o=mat(d, d), self_o_b=zeros,
                 cross_ln_w=ones, cross_ln_b=zeros, cross_q=mat(d, d), cross_q_b=zeros, cross_k=mat(d, d),
                 cross_v=mat(d, d), cross_v_b=zeros, cross_o=mat(d, d), cross_o_b=zeros,
                 mlp_ln_w=ones, mlp_ln_b=zeros, mlp0=mat(4 * d, d), mlp0_b=np.zeros(4 * d, np.float32),
                 mlp2=mat(d, 4 * d), mlp2_b=zeros)
    w = dict(token_embedding=mat(V, d), positional_embedding=small(ctx, d), ln_w=ones, ln_b=zeros, layers=[layer])
    return wgdec.ArrayModel(V, d, H, 1, ctx, w)


@pytest.mark.parametrize("beam", [1, 2])
def test_reference_decoder_tests(kat, beam):
    # internal/model/decoder_test.go:89-180: non-empty segments for greedy / beam 2
    c = kat["decoder_tests"]
    m = reference_test_model(kat)
    dec = wgdec.WhisperDecoder(m)
    enc = np.full((c["enc_len"], c["d"]), c["enc_value"], np.float32)
    params = wgdec.DecoderParams(prompt=c["prompt"], beam_size=beam, max_tokens=c["greedy_max_tokens"],
                                 temperature=c["temperature"], mode=wgdec.MODE_REF_COMPAT)
    segs = dec.decode(enc, params)
    assert len(segs) == 1 and len(segs[0].tokens) > 0
    gt, gl, _ = dec.decode_tokens([enc], params)
    rt, rl, _ = oracle.decode(m, [enc], params, c["ctx"])
    assert gt[0, :gl[0]].tolist() == rt[0, :rl[0]].tolist()
    dec.close()


def test_context_cancellation(kat, tiny):
    # internal/model/decoder_test.go:125-152: a cancelled ctx errors with context.Canceled
    m, dec = tiny
    ctx = wgdec.Context()
    ctx.cancel()
    with pytest.raises(wgdec.DecodeError) as ei:
        dec.decode(m.encoder_output(0), wgdec.DecoderParams(prompt=PROMPT, max_tokens=10), ctx)
    assert wgdec.is_canceled(ei.value)


def test_cancel_during_decode(tiny):
    m, dec = tiny
    ctx = wgdec.Context()
    threading.Timer(0.05, ctx.cancel).start()
    with pytest.raises(wgdec.DecodeError) as ei:
        for _ in range(1000):
            dec.decode(m.encoder_output(0), wgdec.DecoderParams(prompt=PROMPT, max_tokens=200), ctx)
    assert wgdec.is_canceled(ei.value)


@pytest.mark.parametrize("qtype", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"])
def test_teacher_forced_tensor_core_path(qtype):
    """50 utterances (R = 50 > 16): every GEMM of the step, the cross K/V
    precompute and the logits run on the tcgen05 kernel (dequantised tiles in
    tensor memory), with all epilogue modes (QKV scatter, residual add, GELU,
    cross K/V scatter), for each quantisation type."""
    m = wgdec.SyntheticModel(51864, 256, 4, 2, 448, qtype, seed=23)
    dec = wgdec.WhisperDecoder(m)
    try:
        U, T = 50, 64
        encs = [m.encoder_output(u, T) for u in range(U)]
        forced = np.random.default_rng(5).integers(0, 50257, size=(U, 3))
        gpu = dec.teacher_forced_logits(encs, PROMPT, forced, wgdec.MODE_CORRECT)
        for u in range(U):
            ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], wgdec.MODE_CORRECT, m.n_vocab)
            assert_logits_close(gpu[:, u, :], ref)
    finally:
        dec.close()
        m.close()


_LN_FUSE_SCRIPT = r"""
import sys, numpy as np
sys.path[:0] = [{pkg!r}]
import wgdec
m = wgdec.SyntheticModel(51864, {d}, {d} // 64, 2, 448, "Q8_0", seed=31)
dec = wgdec.WhisperDecoder(m)
encs = [m.encoder_output(u, 96) for u in range(2)]
forced = np.random.default_rng(3).integers(0, 50257, size=(2, 3))
np.save({out!r}, dec.teacher_forced_logits(encs, [50258, 50259, 50357, 50363], forced, wgdec.MODE_CORRECT))
"""


@pytest.mark.parametrize("d", [256, 384])
def test_fused_input_layernorm(tmp_path, d):
    """The small-batch GEMV's own LayerNorm (WG_LN_FUSE=1, the default) keeps
    the normalised activations as f16 high + low parts, the separate
    LayerNorm kernel (WG_LN_FUSE=0) rounds them to f16 once: both meet the
    gate, and the fused path is the closer one to the oracle (lane-strided
    d = 256 and float4 d = 384 summation orders)."""
    import os
    import subprocess
    import sys
    outs = {}
    for fuse in ("0", "1"):
        out = tmp_path / ("logits_%s.npy" % fuse)
        code = _LN_FUSE_SCRIPT.format(pkg=str(wgdec.PKG), d=d, out=str(out))
        env = dict(os.environ, WG_LN_FUSE=fuse)
        subprocess.run([sys.executable, "-c", code], env=env, check=True, timeout=300)
        outs[fuse] = np.load(out)
    m = wgdec.SyntheticModel(51864, d, d // 64, 2, 448, "Q8_0", seed=31)
    encs = [m.encoder_output(u, 96) for u in range(2)]
    forced = np.random.default_rng(3).integers(0, 50257, size=(2, 3))
    errs = {}
    for fuse, g in outs.items():
        e = 0.0
        for u in range(2):
            ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], wgdec.MODE_CORRECT, m.n_vocab)
            assert_logits_close(g[:, u, :], ref)
            e = max(e, float(np.sqrt(np.mean((g[:, u, :].astype(np.float64) - ref) ** 2))))
        errs[fuse] = e
    m.close()
    assert errs["1"] <= errs["0"], errs
