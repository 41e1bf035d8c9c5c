"""Host-side logic of the drop-in that needs no GPU: the text post-processing
and retry test of the reference decoder (decoder.go:1170-1230, :1415-1459),
mirrored in wgdec for the retry loop around the device decode."""
import wgdec


class Vocab:
    """A stand-in vocabulary: token t -> text[t] (vocab.Vocabulary's Decode / DecodeToken)."""

    def __init__(self, texts, eot=-1):
        self.texts, self.eot = texts, eot

    def decode_token(self, t):
        return self.texts.get(t, "")

    def decode(self, ids):
        return "".join(self.texts.get(t, "") for t in ids)


def test_collapse_repeated_substrings():
    f = wgdec.collapse_repeated_substrings
    assert f("tra tra tra tra", 6, 3) == "tra tra"
    assert f("aaaa", 6, 3) == "aa"
    assert f("abcabcabc!", 6, 3) == "abc!"
    assert f("hello", 6, 3) == "hello"
    assert f("", 6, 3) == "" and f("xx", 0, 3) == "xx" and f("xxx", 6, 1) == "xxx"


def test_compression_ratio():
    assert wgdec.compression_ratio("") == 0.0
    assert wgdec.compression_ratio("ab" * 200) > 2.4          # a decoding loop: retried
    text = "the quick brown fox jumps over the lazy dog"
    assert wgdec.compression_ratio(text) < 2.4                 # ordinary text: kept


def test_tokens_to_segments_with_vocabulary():
    v = Vocabulary = Vocab({10: " tra", 11: " la", 12: "!"})
    segs = wgdec.tokens_to_segments([1, 2, 10, 10, 10, 11, 12], [1, 2], v)
    assert len(segs) == 1
    # consecutive identical token texts are collapsed (decoder.go:1433-1437)
    assert [t.id for t in segs[0].tokens] == [10, 11, 12]
    assert segs[0].text == " tra la!"
    assert wgdec.tokens_to_segments([1, 2], [1, 2], v) == []
    assert [t.id for t in wgdec.tokens_to_segments([1, 5, 5], [1])[0].tokens] == [5, 5]  # no vocabulary
