"""The temperature schedule with the compression-ratio retry and the
vocabulary's EOT (decoder.go:433-515 greedy, :536-716 beam, :1170-1183,
SetVocabulary :85-95), run by the host mirror around device decodes.

An utterance whose decoded text compresses by more than 2.4 is decoded again
at temperature + 0.2 * attempt, up to 3 attempts, unless NoFallback; the
result is the last attempt's. Stand-in vocabularies make the text
repetitive (every token "abcd": always retried) or not (distinct random
text per token: never retried)."""
import numpy as np
import pytest

import wgdec

pytestmark = pytest.mark.gpu
PROMPT = [50258, 50259, 50357, 50363]


class Vocab:
    def __init__(self, text_of, eot=-1):
        self.text_of, self.eot = text_of, eot

    def decode_token(self, t):
        return self.text_of(t)

    def decode(self, ids):
        return "".join(self.text_of(t) for t in ids)


@pytest.fixture
def model():
    m = wgdec.SyntheticModel(51864, 384, 6, 2, 448, "Q8_0", seed=61)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


def _tokens(segs):
    return [t.id for t in segs[0].tokens] if segs else []


@pytest.mark.parametrize("beam", [1, 5])
def test_repetitive_text_is_decoded_again_at_higher_temperature(model, beam):
    m, dec = model
    encs = [m.encoder_output(u, 200) for u in range(2)]
    base = wgdec.DecoderParams(prompt=PROMPT, beam_size=beam, max_tokens=100, suppress_eot=True)
    last = dec.decode_tokens(encs, wgdec.DecoderParams(**{**base.__dict__, "attempt": 2}))
    dec.set_vocabulary(Vocab(lambda t: "abcd"))
    assert wgdec.compression_ratio("abcd" * 100) > 2.4
    segs = dec.decode_batch(encs, base)
    for u in range(2):
        # consecutive tokens with the same text are dropped from the segment
        # (decoder.go:1433-1437): compare with the attempt-2 decode filtered alike
        want = last[0][u, len(PROMPT):last[1][u]].tolist()[:1]
        assert _tokens(segs[u]) == want
        assert segs[u][0].text == "abcd"
    nof = dec.decode_batch(encs, wgdec.DecoderParams(**{**base.__dict__, "no_fallback": True}))
    first = dec.decode_tokens(encs, base)
    for u in range(2):
        assert _tokens(nof[u])[:1] == first[0][u, len(PROMPT):len(PROMPT) + 1].tolist()


def test_ordinary_text_is_kept(model):
    m, dec = model
    rng = np.random.default_rng(0)
    words = {}

    def text_of(t):
        if t not in words:
            words[t] = "".join(chr(97 + c) for c in rng.integers(0, 26, size=5)) + " "
        return words[t]
    encs = [m.encoder_output(7, 200)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=5, max_tokens=30, suppress_eot=True)
    toks, lens, _ = dec.decode_tokens(encs, params)
    dec.set_vocabulary(Vocab(text_of))
    segs = dec.decode(encs[0], params)
    gen = toks[0, len(PROMPT):lens[0]].tolist()
    assert [t.id for t in segs[0].tokens] == [t for i, t in enumerate(gen) if i == 0 or text_of(t) != text_of(gen[i - 1])]


def test_vocabulary_eot_stops_the_decode(model):
    m, dec = model
    enc = m.encoder_output(3, 200)
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=1, max_tokens=10)
    toks, lens, _ = dec.decode_tokens([enc], params)
    first = int(toks[0, len(PROMPT)])
    dec.set_vocabulary(Vocab(lambda t: "x%d " % t, eot=first))
    toks2, lens2, _ = dec.decode_tokens([enc], params)
    assert lens2[0] == len(PROMPT) + 1 and toks2[0, len(PROMPT)] == first
