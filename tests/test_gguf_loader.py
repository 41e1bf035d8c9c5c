"""wg_model_create_from_gguf: the decoder's weights from a GGUF model file
(internal/gguf/gguf.go:52-134, internal/model/decoder.go:97-303,
internal/model/compat.go:31-148).

CPU part: files written in the reference writer's layout parse, resolve
under whisper.cpp and Hugging Face names, and reach the device step (which
reports that no device is present here); malformed files fail with the
reference's error texts. GPU part: a decoder loaded from the file gives
bit-identical logits to one created from the same weights in memory."""
import ctypes

import numpy as np
import pytest

import gguf_writer
import wgdec

ERR_INVALID, ERR_NO_DEVICE = 1, 8


def _create(path):
    h = ctypes.c_void_p()
    rc = wgdec.lib().wg_model_create_from_gguf(str(path).encode(), None, 0, ctypes.byref(h))
    if rc == 0:
        wgdec.lib().wg_model_destroy(h)
    return rc, wgdec.last_error()


@pytest.fixture(scope="module")
def model():
    m = wgdec.SyntheticModel(1000, 128, 2, 2, 448, "Q5_1", seed=3)
    yield m
    m.close()


def _no_gpu():
    return wgdec.device_count() == 0


@pytest.mark.parametrize("names,f16,meta", [("whisper.cpp", False, True), ("hf", False, True),
                                            ("whisper.cpp", True, False), ("hf", True, False)])
def test_parses_and_resolves(tmp_path, model, names, f16, meta):
    if not _no_gpu():
        pytest.skip("CPU-side check: with a device the model is created (GPU test below)")
    p = tmp_path / "m.gguf"
    gguf_writer.write(p, model, names=names, f16_vectors=f16, meta=meta, vocab_tokens=50)
    rc, msg = _create(p)
    assert rc == ERR_NO_DEVICE, msg  # every tensor was found and validated; only the upload is left


def test_malformed_files(tmp_path, model):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + b"\0" * 64)
    assert _create(p) == (ERR_INVALID, "gguf: invalid magic")
    p.write_bytes(b"GGUF" + (7).to_bytes(4, "little") + b"\0" * 16)
    rc, msg = _create(p)
    assert rc == ERR_INVALID and msg.startswith("gguf: unsupported version")
    gguf_writer.write(p, model)
    raw = p.read_bytes()
    p.write_bytes(raw[:len(raw) // 2])  # tensor data cut off
    rc, msg = _create(p)
    assert rc == ERR_INVALID and "decoder" in msg
    rc, msg = _create(tmp_path / "missing.gguf")
    assert rc == ERR_INVALID and msg.startswith("gguf: open")


@pytest.mark.gpu
@pytest.mark.parametrize("names", ["whisper.cpp", "hf"])
def test_gguf_model_matches_in_memory_model(tmp_path, names):
    m = wgdec.SyntheticModel(51864, 384, 6, 2, 448, "Q8_0", seed=77)
    p = tmp_path / "m.gguf"
    gguf_writer.write(p, m, names=names, vocab_tokens=100)
    a = wgdec.WhisperDecoder(m)
    b = wgdec.WhisperDecoder.from_gguf(p)
    try:
        assert a.weight_bytes() == b.weight_bytes()
        enc = m.encoder_output(1, 128)
        forced = np.random.default_rng(2).integers(0, 50257, size=6)
        la = a.teacher_forced_logits(enc, [50258, 50259, 50357, 50363], forced)
        lb = b.teacher_forced_logits(enc, [50258, 50259, 50357, 50363], forced)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    finally:
        a.close()
        b.close()
        m.close()
