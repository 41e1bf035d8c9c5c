"""Decoder parity at the benchmark's shapes and row counts, through the C ABI.

The other decoder tests use small models and at most 20 rows per step. This
file runs the kernels the benchmark itself runs, against the CPU oracle:

* teacher-forced logits at the shape and quantisation of every BASELINE
  configuration (configs 1-4 in full; config 5, large-v3-shaped, with 4 of
  its 32 layers), 200 forced tokens so the f16 KV cache is read out to
  position 203 (the bench decodes positions 3..227);
* batched teacher forcing at config 5 / config 4 widths with 32, 40 and 56
  rows per step (tcgen05 GEMMs, the 4-warp self-attention kernel from 512
  (row, head) pairs on, the streaming cross-attention kernel);
* greedy decoding with 72 rows (the one-CTA-per-row greedy kernel above 64
  rows) and beam-5 decoding of 14 utterances (70 rows: the one-CTA top-k
  kernel, the beam merge of 14 utterances), compared step by step;
* the reference's edge cases: language detection (Prompt = [SOT],
  MaxTokens = 1, pipeline.go:243-252), the >20 repeat stop
  (decoder.go:475-484, :675-691) and SuppressNST with a finite
  NoSpeechThold (decoder.go:1016-1034).

Gates (north star): teacher-forced logits within max-abs 2e-2 AND rel 1e-3,
both asserted for every step, rel read as max|gpu - ref| / max|ref|. Token
decisions: the GPU must make the oracle's decision at every step whose
decision margin exceeds the 2e-2 logit tolerance. The decodes are compared
step by step; where they first differ, the oracle's margin at that step must
be <= 2e-2 (a near-tie the tolerance allows either way), and the comparison
of that utterance ends there. The margin is the top-2 logit gap for greedy;
for beam search the smallest of every live row's 5th/6th logit gap and the
gaps among the best B+1 candidates' normalised scores (the 5th/6th
candidate boundary, and the order of the kept beams).
"""
import os

import numpy as np
import pytest

import oracle
import wgdec

pytestmark = pytest.mark.gpu
ATOL, REL = 2e-2, 1e-3
MARGIN = 2e-2  # token decisions are compared wherever the oracle's margin exceeds this
PROMPT = [50258, 50259, 50357, 50363]
THREADS = os.cpu_count() or 1

# (name, vocab, d, heads, layers, qtype) of BASELINE.json configs 1-5
CONFIGS = {
    "c1": (51864, 384, 6, 4, "Q8_0"),
    "c2": (51865, 512, 8, 6, "Q4_0"),
    "c3": (51865, 768, 12, 12, "Q5_1"),
    "c4": (51865, 1024, 16, 24, "Q5_0"),
    "c5": (51866, 1280, 20, 4, "Q8_0"),  # 4 of large-v3's 32 layers
}


@pytest.fixture(scope="module", autouse=True)
def _oracle_threads():
    oracle.set_threads(THREADS)
    yield
    oracle.set_threads(1)


def gate(gpu, ref, what=""):
    """Both gates on every step (row of logits)."""
    gpu = np.asarray(gpu).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref).reshape(-1, ref.shape[-1])
    worst = 0.0
    for s in range(ref.shape[0]):
        err = float(np.max(np.abs(gpu[s] - ref[s])))
        scale = float(np.max(np.abs(ref[s])))
        assert err <= ATOL, "%s step %d: max abs err %.3g > %g" % (what, s, err, ATOL)
        assert err <= REL * scale, "%s step %d: max abs err %.3g > %g * max|ref| (%.3g)" % (what, s, err, REL,
                                                                                            scale)
        worst = max(worst, err)
    return worst


def synthetic(name, layers=None, seed=20261201):
    V, d, H, L, qt = CONFIGS[name]
    return wgdec.SyntheticModel(V, d, H, layers or L, 448, qt, seed=seed)


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_teacher_forced_config_shapes(name):
    """One utterance (the batch-1 kernels: small-batch GEMV with the fused
    LayerNorm, cluster cross-attention, single-round self-attention), 200
    forced tokens uniform in [0, 50256], 1500 encoder frames."""
    m = synthetic(name)
    dec = wgdec.WhisperDecoder(m)
    try:
        enc = m.encoder_output(3)
        forced = np.random.default_rng(17).integers(0, 50257, size=200)
        gpu = dec.teacher_forced_logits(enc, PROMPT, forced, wgdec.MODE_CORRECT)[:, 0, :]
        ref = oracle.teacher_forced(m, enc, PROMPT, forced, wgdec.MODE_CORRECT, m.n_vocab)
        gate(gpu, ref, name)
    finally:
        dec.close()
        m.close()


def test_teacher_forced_ref_compat_config_shape():
    """REF_COMPAT semantics (no prefill, only KV slot 0 visible) at config 3's shape."""
    m = synthetic("c3")
    dec = wgdec.WhisperDecoder(m)
    try:
        enc = m.encoder_output(4)
        forced = np.random.default_rng(18).integers(0, 50257, size=40)
        gpu = dec.teacher_forced_logits(enc, PROMPT, forced, wgdec.MODE_REF_COMPAT)[:, 0, :]
        ref = oracle.teacher_forced(m, enc, PROMPT, forced, wgdec.MODE_REF_COMPAT, m.n_vocab)
        gate(gpu, ref, "c3 ref_compat")
    finally:
        dec.close()
        m.close()


@pytest.mark.parametrize("name,U,n,check", [("c5", 32, 48, (0, 13, 31)), ("c4", 40, 24, (0, 39)),
                                             ("c5", 56, 24, (0, 55))])
def test_teacher_forced_batched_rows(name, U, n, check):
    """U rows per step at config 5 / config 4 widths: every matmul on the
    tcgen05 kernel with LayerNorm kernels between (the small-batch GEMV takes
    at most 16 rows by default); self-attention on the 4-warp kernel (R * H >= 512),
    cross-attention on the streaming kernel (U * H >= 64). All U rows run on
    the GPU; a few are checked against the oracle (each costs a full CPU
    decode)."""
    m = synthetic(name, layers=4 if name == "c5" else None)
    dec = wgdec.WhisperDecoder(m)
    try:
        encs = [m.encoder_output(100 + u) for u in range(U)]
        forced = np.random.default_rng(U).integers(0, 50257, size=(U, n))
        gpu = dec.teacher_forced_logits(encs, PROMPT, forced, wgdec.MODE_CORRECT)
        for u in check:
            ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], wgdec.MODE_CORRECT, m.n_vocab)
            gate(gpu[:, u, :], ref, "%s row %d" % (name, u))
    finally:
        dec.close()
        m.close()


def test_beam_decode_config3_shape():
    """Config 3's shape and quantisation (d 768, 12 heads, 12 layers, Q5_1,
    odd vocabulary) with beam 5 at one utterance: the batch-1 kernels through
    the job API and the CUDA graph for a full 224-step decode, twice. Every
    token must be in the vocabulary and the two decodes identical (a race in
    a kernel shows up as a difference, or as garbage tokens); the first steps
    are compared with the oracle beam by beam."""
    m = synthetic("c3")
    dec = wgdec.WhisperDecoder(m)
    try:
        enc = m.encoder_output(5)
        params = wgdec.DecoderParams(prompt=PROMPT, beam_size=5, max_tokens=224, suppress_eot=True,
                                     mode=wgdec.MODE_CORRECT)
        t1, l1, s1 = dec.decode_tokens([enc], params)
        t2, l2, s2 = dec.decode_tokens([enc], params)
        n = int(l1[0])
        assert len(PROMPT) < n <= len(PROMPT) + 224
        assert np.all((t1[0, :n] >= 0) & (t1[0, :n] < m.n_vocab))
        np.testing.assert_array_equal(l1, l2)
        np.testing.assert_array_equal(t1, t2)
        np.testing.assert_array_equal(s1, s2)
        assert np.isfinite(s1[0])
        B, M = 5, 6
        short = wgdec.DecoderParams(prompt=PROMPT, beam_size=B, max_tokens=M, suppress_eot=True,
                                    mode=wgdec.MODE_CORRECT)
        tr = oracle.decode_trace(m, [enc], short, m.n_ctx, threads=THREADS)
        job = wgdec.Job(dec, 1, enc.shape[0], short)
        try:
            job.upload([enc])
            job.start()
            for st in range(M):
                done = job.step(1)
                toks, lens, scores = job.beams()
                if st >= tr["steps"][0]:
                    break
                same = lens[0].tolist() == tr["beams_lens"][0, st].tolist() and all(
                    toks[0, b, :lens[0, b]].tolist() == tr["beams_tokens"][0, st, b, :lens[0, b]].tolist()
                    for b in range(B))
                if not same:
                    assert tr["margins"][0, st] <= MARGIN, \
                        "step %d: beams differ at margin %.3g" % (st, tr["margins"][0, st])
                    break
                np.testing.assert_allclose(scores[0], tr["beams_scores"][0, st], atol=2e-2)
                if done:
                    break
        finally:
            job.close()
    finally:
        dec.close()
        m.close()


# ---- token decisions at many rows ------------------------------------------------------
@pytest.fixture(scope="module")
def wide():
    """d = 512, 8 heads, 2 layers, Q8_0, full vocabulary; 64 encoder frames."""
    m = wgdec.SyntheticModel(51864, 512, 8, 2, 448, "Q8_0", seed=41)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


def agree_greedy(gpu_toks, tr, u, P):
    """Number of generated tokens on which the GPU and the oracle agree; a
    first difference must sit at a step whose oracle margin is <= MARGIN."""
    n = int(tr["steps"][u])
    for s in range(n):
        if gpu_toks[P + s] != tr["tokens"][u, P + s]:
            assert tr["margins"][u, s] <= MARGIN, \
                "utterance %d step %d: tokens differ at margin %.3g" % (u, s, tr["margins"][u, s])
            return s
    return n


def test_wide_model_logit_error(wide):
    """The logit error behind the token comparisons, on this model."""
    m, dec = wide
    encs = [m.encoder_output(u, 64) for u in range(2)]
    forced = np.random.default_rng(3).integers(0, 50257, size=(2, 24))
    gpu = dec.teacher_forced_logits(encs, PROMPT, forced, wgdec.MODE_CORRECT)
    for u in range(2):
        ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], wgdec.MODE_CORRECT, m.n_vocab)
        gate(gpu[:, u, :], ref, "wide row %d" % u)


def test_greedy_many_rows(wide):
    """72 utterances greedy (the one-CTA-per-row greedy kernel above 64 rows;
    self-attention on the 4-warp kernel at 72 x 8 >= 512 pairs)."""
    m, dec = wide
    U, M = 72, 24
    encs = [m.encoder_output(u, 64) for u in range(U)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=1, max_tokens=M, mode=wgdec.MODE_CORRECT)
    gt, gl, _ = dec.decode_tokens(encs, params)
    tr = oracle.decode_trace(m, encs, params, m.n_ctx, threads=THREADS)
    P, agreed, full = len(PROMPT), 0, 0
    for u in range(U):
        k = agree_greedy(gt[u], tr, u, P)
        agreed += k
        if k == tr["steps"][u]:
            full += 1
            assert gl[u] == tr["lens"][u]
    assert full >= U * 3 // 4, "only %d of %d utterances decoded identically" % (full, U)


def test_beam_many_rows_step_by_step(wide):
    """14 utterances x beam 5 = 70 rows (the one-CTA top-k kernel above 64
    rows; the beam merge of 14 utterances). After every step the GPU's beams
    (tokens, order, scores) must equal the oracle's; where they first differ,
    that step's oracle margin must be <= MARGIN (a candidate set, kept /
    dropped boundary or beam order decided by a near-tie)."""
    m, dec = wide
    U, B, M = 14, 5, 16
    encs = [m.encoder_output(200 + u, 64) for u in range(U)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=B, max_tokens=M, mode=wgdec.MODE_CORRECT)
    tr = oracle.decode_trace(m, encs, params, m.n_ctx, threads=THREADS)
    job = wgdec.Job(dec, U, 64, params)
    live = [True] * U
    compared = 0
    try:
        job.upload(encs)
        job.start()
        for s in range(M):
            done = job.step(1)
            toks, lens, scores = job.beams()
            for u in range(U):
                if not live[u] or s >= tr["steps"][u]:
                    continue
                same = lens[u].tolist() == tr["beams_lens"][u, s].tolist() and all(
                    toks[u, b, :lens[u, b]].tolist() == tr["beams_tokens"][u, s, b, :lens[u, b]].tolist()
                    for b in range(B))
                if not same:
                    assert tr["margins"][u, s] <= MARGIN, \
                        "utterance %d step %d: beams differ at margin %.3g" % (u, s, tr["margins"][u, s])
                    live[u] = False
                    continue
                np.testing.assert_allclose(scores[u], tr["beams_scores"][u, s], atol=2e-2)
                compared += 1
            if done:
                break
    finally:
        job.close()
    assert compared >= U * M // 2, "only %d (utterance, step) pairs agreed" % compared


# ---- reference edge cases ---------------------------------------------------------------------
def test_language_detection_call(wide):
    """detectLanguage's Decode call: Prompt = [SOT], MaxTokens = 1, greedy (pipeline.go:243-252)."""
    m, dec = wide
    encs = [m.encoder_output(u, 64) for u in range(3)]
    params = wgdec.DecoderParams(prompt=[50258], beam_size=1, max_tokens=1, mode=wgdec.MODE_CORRECT)
    gt, gl, _ = dec.decode_tokens(encs, params)
    tr = oracle.decode_trace(m, encs, params, m.n_ctx, threads=THREADS)
    for u in range(3):
        assert gl[u] == tr["lens"][u] == 2
        agree_greedy(gt[u], tr, u, 1)
    segs = dec.decode(encs[0], params)
    assert len(segs) == 1 and len(segs[0].tokens) == 1


def repeat_model(d=64, V=512, big=1.0):
    """A one-layer F32 decoder whose every matrix is zero, so x = E[token]
    after the embedding and the logits are LayerNorm(E[token]) . E^T: token 7
    has a large zero-mean row, so after token 7 it wins by ~big * d, more than
    the repetition penalty removes in 21 steps (2 per occurrence)."""
    rng = np.random.default_rng(5)
    E = (rng.standard_normal((V, d)) * 0.02).astype(np.float32)
    v = rng.standard_normal(d).astype(np.float32)
    v -= v.mean()
    v /= v.std()
    E[7] = big * v
    z = lambda *s: np.zeros(s, np.float32)
    mat = lambda r, k: ("F32", r, k, z(r, k))
    ones = np.ones(d, np.float32)
    layer = dict(self_ln_w=ones, self_ln_b=z(d), self_q=mat(d, d), self_q_b=z(d), self_k=mat(d, d),
                 self_v=mat(d, d), self_v_b=z(d), self_o=mat(d, d), self_o_b=z(d),
                 cross_ln_w=ones, cross_ln_b=z(d), cross_q=mat(d, d), cross_q_b=z(d), cross_k=mat(d, d),
                 cross_v=mat(d, d), cross_v_b=z(d), cross_o=mat(d, d), cross_o_b=z(d),
                 mlp_ln_w=ones, mlp_ln_b=z(d), mlp0=mat(4 * d, d), mlp0_b=z(4 * d),
                 mlp2=mat(d, 4 * d), mlp2_b=z(d))
    w = dict(token_embedding=("F32", V, d, E), positional_embedding=z(448, d), ln_w=ones, ln_b=z(d),
             layers=[layer])
    return wgdec.ArrayModel(V, d, 1, 1, 448, w, eot=V - 1)


@pytest.mark.parametrize("beam", [1, 5])
def test_repeat_stop(beam):
    """Token 7 repeats: greedy stops after 21 identical generated tokens
    (streak > 20, decoder.go:475-484); beam search stops once the best beam
    ends in more than 20 identical tokens (decoder.go:675-691)."""
    m = repeat_model()
    dec = wgdec.WhisperDecoder(m)
    try:
        enc = np.zeros((16, 64), np.float32)
        params = wgdec.DecoderParams(prompt=[7], beam_size=beam, max_tokens=100, mode=wgdec.MODE_CORRECT)
        gt, gl, _ = dec.decode_tokens([enc], params)
        rt, rl, _ = oracle.decode(m, [enc], params, 448)
        assert gl[0] == rl[0] < 1 + 100
        assert gt[0, :gl[0]].tolist() == rt[0, :rl[0]].tolist()
        assert gt[0, 1:gl[0]].tolist().count(7) >= 20
    finally:
        dec.close()


@pytest.mark.parametrize("below", [True, False])
def test_suppress_nst_finite_threshold(wide, below):
    """SuppressNST with a finite NoSpeechThold (decoder.go:1016-1034): the
    model's EOT id is set to the token the oracle picks at the first step; with
    logits[eot] < -NoSpeechThold the greedy pick moves to the best other token,
    otherwise EOT is taken and the decode ends."""
    m0, _ = wide
    enc = m0.encoder_output(9, 64)
    p0 = wgdec.DecoderParams(prompt=PROMPT, beam_size=1, max_tokens=1, mode=wgdec.MODE_CORRECT)
    first = int(oracle.decode(m0, [enc], p0, 448)[0][0, len(PROMPT)])
    lg = oracle.teacher_forced(m0, enc, PROMPT, [first], wgdec.MODE_CORRECT, m0.n_vocab)[0]
    lg = oracle.apply_penalty(lg, PROMPT)
    m = wgdec.SyntheticModel(51864, 512, 8, 2, 448, "Q8_0", seed=41)
    m.desc.contents.eot = first
    dec = wgdec.WhisperDecoder(m)
    try:
        # -thold sits 0.5 above (below: EOT is suppressed) or under the EOT logit
        thold = -(lg[first] + 0.5) if below else -(lg[first] - 0.5)
        params = wgdec.DecoderParams(prompt=PROMPT, beam_size=1, max_tokens=6, suppress_nst=True,
                                     no_speech_thold=float(thold), mode=wgdec.MODE_CORRECT)
        gt, gl, _ = dec.decode_tokens([enc], params)
        tr = oracle.decode_trace(m, [enc], params, 448, threads=THREADS)
        P = len(PROMPT)
        assert tr["margins"][0, 0] > MARGIN  # the first decision is clear-cut by construction
        assert agree_greedy(gt[0], tr, 0, P) >= 1
        if below:
            assert gt[0, P] != first
        else:
            assert gt[0, P] == first and gl[0] == P + 1
    finally:
        dec.close()
        m.close()
