"""C-ABI boundary checks that need no GPU.

* every function include/wg_decoder.h declares is exported by libwgdec.so
  (the symbols a cgo binding of internal/cuda links against);
* argument validation and the no-device path return the documented status
  codes and messages (the reference's error texts where it has one);
* the host-side mirror of the reference API (wgdec) maps DecoderParams the
  way internal/model/decoder.go reads them.
"""
import ctypes
import re

import numpy as np
import pytest

import wgdec
from conftest import ROOT

HEADER = ROOT / "include" / "wg_decoder.h"
ERR_INVALID = 1    # WG_ERR_INVALID
ERR_NO_DEVICE = 8  # WG_ERR_NO_DEVICE


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|void)\s+(wg_[a-z0-9_]+)\s*\(", text, re.M)))


def no_device():
    n = ctypes.c_int(-1)
    assert wgdec.lib().wg_device_count(ctypes.byref(n)) == 0
    return n.value == 0


def last_error():
    buf = ctypes.create_string_buffer(512)
    wgdec.lib().wg_last_error(buf, len(buf))
    return buf.value.decode()


def test_header_declares_the_api():
    names = declared_functions()
    for n in ("wg_model_create", "wg_job_create", "wg_job_step", "wg_job_result", "wg_decode",
              "wg_teacher_forced_logits", "wg_dequant_test", "wg_matmul_test", "wg_last_error"):
        assert n in names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(wgdec.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_launch_counter_and_error_buffer():
    n = ctypes.c_int64(-1)
    assert wgdec.lib().wg_kernel_launch_count(ctypes.byref(n)) == 0
    assert n.value >= 0
    assert wgdec.lib().wg_last_error(None, 0) == 0


def test_null_arguments_are_rejected():
    L = wgdec.lib()
    out = ctypes.c_void_p()
    assert L.wg_model_create(None, None, 0, ctypes.byref(out)) == ERR_INVALID
    assert "null argument" in last_error()
    assert L.wg_job_create(None, 1, 1500, None, 0, None, ctypes.byref(out)) == ERR_INVALID
    buf = np.zeros(4, np.float32)
    assert L.wg_dequant_test(8, None, 32, buf.ctypes.data_as(ctypes.POINTER(ctypes.c_float))) == ERR_INVALID
    assert L.wg_model_destroy(None) == 0
    assert L.wg_job_destroy(None) == 0


def test_invalid_hyper_parameters_use_the_reference_message():
    desc = wgdec.WgModelDesc()
    desc.n_vocab, desc.n_state, desc.n_head, desc.n_layer, desc.n_text_ctx = 100, 30, 4, 1, 16  # 30 % 4 != 0
    out = ctypes.c_void_p()
    rc = wgdec.lib().wg_model_create(ctypes.byref(desc), None, 0, ctypes.byref(out))
    assert rc == ERR_INVALID
    assert last_error().startswith("model: decoder: invalid hyper-parameters")


@pytest.mark.skipif(not no_device(), reason="a CUDA device is visible")
def test_no_device_is_reported_not_worked_around():
    """No CPU fallback: without a GPU the library refuses with WG_ERR_NO_DEVICE."""
    m = wgdec.SyntheticModel(64, 64, 1, 1, 16, "Q8_0", seed=3)
    try:
        with pytest.raises(wgdec.DecodeError) as ei:
            wgdec.WhisperDecoder(m)
        assert ei.value.status == ERR_NO_DEVICE
        raw = np.frombuffer(wgdec.quantize("Q8_0", np.ones(64, np.float32)), dtype=np.uint8).copy()
        out = np.zeros(64, np.float32)
        rc = wgdec.lib().wg_dequant_test(8, raw.ctypes.data, 64, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        assert rc == ERR_NO_DEVICE
    finally:
        m.close()


def test_decoder_params_mapping():
    p = wgdec.DecoderParams()
    c = p.to_c()
    # decoder.go:153-171 DefaultDecoderParams: greedy, temperature 0, thresholds
    assert c.beam_size == p.beam_size == 1
    assert c.mode == wgdec.MODE_CORRECT
    # decoder.go:421-430: MaxTokens <= 0 means the text context minus the prompt
    assert wgdec.max_tokens_for(p, 448) == 448
    assert wgdec.max_tokens_for(wgdec.DecoderParams(prompt=[1, 2, 3, 4], max_tokens=500), 448) == 444
    p2 = wgdec.DecoderParams(beam_size=5, temperature=0.0, max_tokens=17, mode=wgdec.MODE_REF_COMPAT,
                             suppress_eot=True)
    c2 = p2.to_c()
    assert (c2.beam_size, c2.max_tokens, c2.mode, c2.suppress_eot) == (5, 17, wgdec.MODE_REF_COMPAT, 1)


def test_noalloc_matmul_rejects_bad_arguments_before_any_device_work():
    """wg_model_matmul_noalloc checks its arguments first: a null model (or a
    bad layer / matrix index) is rejected with WG_ERR_INVALID and a message,
    without touching a device."""
    L = wgdec.lib()
    rc = L.wg_model_matmul_noalloc(None, 0, 0, 0, None, 0, 0, None, 0, None, 1)
    assert rc == ERR_INVALID
    assert last_error() == "wg_model_matmul_noalloc: bad argument"
