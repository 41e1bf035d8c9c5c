"""Pipeline batching (wg_batcher_*): single-utterance Decode calls from many
threads, as the reference's pipeline makes them (internal/model/pipeline.go:
90-193, one Decode per 30-s chunk; concurrent Transcribe calls, whisper.go:24),
gathered into shared GPU jobs. Every caller must get exactly the tokens a
decode of its utterance inside one batched job gives (rows of a job are
computed independently, so a row's result does not depend on its place)."""
import threading

import numpy as np
import pytest

import wgdec

pytestmark = pytest.mark.gpu
PROMPT = [50258, 50259, 50357, 50363]


@pytest.fixture(scope="module")
def model():
    m = wgdec.SyntheticModel(51864, 384, 6, 2, 448, "Q8_0", seed=91)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


def _run_threads(fn, n):
    out, errs = [None] * n, []

    def body(i):
        try:
            out[i] = fn(i)
        except Exception as e:  # re-raised below
            errs.append(e)
    ts = [threading.Thread(target=body, args=(i,)) for i in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    if errs:
        raise errs[0]
    return out


@pytest.mark.parametrize("beam", [1, 5])
def test_concurrent_calls_share_jobs(model, beam):
    m, dec = model
    N = 12
    encs = [m.encoder_output(40 + u, 200) for u in range(N)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=beam, max_tokens=10, suppress_eot=True)
    ref, rl, rs = dec.decode_tokens(encs, params)  # one job of all twelve
    b = wgdec.Batcher(dec, max_utterances=16, window_us=300000)
    try:
        got = _run_threads(lambda i: b.decode_tokens(encs[i], params), N)
        jobs, utts = b.stats()
    finally:
        b.close()
    assert utts == N and jobs < N
    for i in range(N):
        toks, score = got[i]
        assert toks.tolist() == ref[i, :rl[i]].tolist()
        assert score == pytest.approx(float(rs[i]), abs=1e-6)


def test_incompatible_requests_go_to_separate_jobs(model):
    m, dec = model
    encs = [m.encoder_output(70 + u, 200) for u in range(6)]
    p1 = wgdec.DecoderParams(prompt=PROMPT, max_tokens=6, suppress_eot=True)
    p2 = wgdec.DecoderParams(prompt=PROMPT[:3], max_tokens=6, suppress_eot=True)  # a different prompt
    b = wgdec.Batcher(dec, max_utterances=8, window_us=200000)
    try:
        got = _run_threads(lambda i: b.decode_tokens(encs[i], p1 if i % 2 == 0 else p2), 6)
        jobs, utts = b.stats()
    finally:
        b.close()
    assert utts == 6 and jobs >= 2
    r1 = dec.decode_tokens(encs[0::2], p1)
    r2 = dec.decode_tokens(encs[1::2], p2)
    for k, i in enumerate(range(0, 6, 2)):
        assert got[i][0].tolist() == r1[0][k, :r1[1][k]].tolist()
    for k, i in enumerate(range(1, 6, 2)):
        assert got[i][0].tolist() == r2[0][k, :r2[1][k]].tolist()


def test_cancelled_request(model):
    m, dec = model
    b = wgdec.Batcher(dec, max_utterances=4, window_us=1000)
    ctx = wgdec.Context()
    ctx.cancel()
    try:
        with pytest.raises(wgdec.DecodeError) as ei:
            b.decode_tokens(m.encoder_output(0, 200), wgdec.DecoderParams(prompt=PROMPT, max_tokens=200), ctx)
        assert ei.value.status == 5
    finally:
        b.close()
