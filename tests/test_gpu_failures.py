"""Failure handling on the GPU without faulting it.

* Host-side fault injection (WG_FAULT_INJECT=step:N | device:D) ends a decode
  with WG_ERR_INJECTED at that point; the next decode runs normally.
* The host watchdog (WG_TIMEOUT_MS) turns device work that outlasts the
  deadline into WG_ERR_TIMEOUT; the device work still completes and the
  library stays usable.
* A bounded device-side wait that runs out: with WG_TEST_TC_STALL=1 the
  tcgen05 GEMM's activation loader leaves out its first copy (a barrier phase
  that nothing completes), so the MMA issuer's wait expires after
  WG_TEST_WAIT_NS; the kernel raises its abort flag, records the code in its
  error word, lets the copies it issued land, waits for the MMAs it issued,
  frees its tensor memory and returns. The host reports WG_ERR_DEVICE_FLAG,
  and the same process then computes correct results again.

These mirror the reference's error conventions: wrapped errors with the
"model: decode: ..." prefix (decoder.go:442-447) and context.Canceled for
cancellation (decoder_test.go:145-151, covered in test_gpu_decoder.py).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import wgdec

pytestmark = pytest.mark.gpu
PROMPT = [50258, 50259, 50357, 50363]
ERR_TIMEOUT, ERR_INJECTED, ERR_DEVICE_FLAG = 6, 7, 9


@pytest.fixture(scope="module")
def small():
    m = wgdec.SyntheticModel(51864, 384, 6, 2, 448, "Q8_0", seed=13)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


@pytest.fixture
def env(monkeypatch):
    return monkeypatch


def test_fault_injection_at_a_step(small, env):
    m, dec = small
    enc = m.encoder_output(0, 64)
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=1, max_tokens=20)
    env.setenv("WG_FAULT_INJECT", "step:3")
    with pytest.raises(wgdec.DecodeError) as ei:
        dec.decode(enc, params)
    assert ei.value.status == ERR_INJECTED
    assert "injected fault at step 3" in str(ei.value) and str(ei.value).startswith("model: decode:")
    env.delenv("WG_FAULT_INJECT")
    segs = dec.decode(enc, params)
    assert len(segs) == 1 and len(segs[0].tokens) > 0


def test_fault_injection_on_a_device(small, env):
    m, dec = small
    env.setenv("WG_FAULT_INJECT", "device:0")
    with pytest.raises(wgdec.DecodeError) as ei:
        dec.decode(m.encoder_output(1, 64), wgdec.DecoderParams(prompt=PROMPT, max_tokens=4))
    assert ei.value.status == ERR_INJECTED and "device 0" in str(ei.value)
    env.delenv("WG_FAULT_INJECT")
    assert len(dec.decode(m.encoder_output(1, 64), wgdec.DecoderParams(prompt=PROMPT, max_tokens=4))) == 1


def test_watchdog_deadline(small, env):
    """A 1 ms deadline cannot cover a 1500-frame cross K/V precompute plus 100
    token steps of 8 utterances: the wait returns WG_ERR_TIMEOUT."""
    m, dec = small
    encs = [m.encoder_output(u) for u in range(8)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=5, max_tokens=100, suppress_eot=True)
    env.setenv("WG_TIMEOUT_MS", "1")
    with pytest.raises(wgdec.DecodeError) as ei:
        dec.decode_tokens(encs, params)
    assert ei.value.status == ERR_TIMEOUT and "watchdog" in str(ei.value)
    env.delenv("WG_TIMEOUT_MS")
    toks, lens, _ = dec.decode_tokens(encs[:2], wgdec.DecoderParams(prompt=PROMPT, max_tokens=8))
    assert (lens == len(PROMPT) + 8).all() or (lens > len(PROMPT)).all()


_STALL_SCRIPT = r"""
import os, sys, numpy as np
sys.path[:0] = [{pkg!r}, {orc!r}]
import wgdec, oracle
oracle.set_threads(os.cpu_count() or 1)
rng = np.random.default_rng(1)
out = {{}}
# (40 weight groups x 4 row tiles fill the GPU: no K split) and (10 groups:
# K split over a 7-CTA cluster, partial tiles in the workspace)
for name, R, rows, K in [("unsplit", 1024, 5120, 1280), ("split", 40, 1280, 1280)]:
    w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    a = rng.standard_normal((R, K)).astype(np.float32)
    raw = wgdec.quantize_matrix("Q8_0", w)
    os.environ["WG_TEST_TC_STALL"] = "1"
    os.environ["WG_TEST_WAIT_NS"] = "20000000"
    try:
        wgdec.matmul("Q8_0", raw, rows, K, a, path=3)
        out[name] = "no error"
    except wgdec.DecodeError as e:
        out[name] = "%d %s" % (e.status, e)
    del os.environ["WG_TEST_TC_STALL"], os.environ["WG_TEST_WAIT_NS"]
    got = wgdec.matmul("Q8_0", raw, rows, K, a, path=3)
    ref = oracle.matmul("Q8_0", raw, rows, K, a)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    out[name + "_after"] = bool(np.max(np.abs(got - ref)) <= 5e-3 * rms)
print(repr(out))
"""


def test_bounded_wait_expiry_in_the_tensor_core_gemm():
    """Run in a child process: the stall and the short wait bound are read
    from its environment at every launch of the tcgen05 kernel."""
    pkg = str(wgdec.PKG)
    orc = str(wgdec.ROOT / "oracle")
    r = subprocess.run([sys.executable, "-c", _STALL_SCRIPT.format(pkg=pkg, orc=orc)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = eval(r.stdout.strip().splitlines()[-1])
    for name in ("unsplit", "split"):
        assert out[name].startswith("%d " % ERR_DEVICE_FLAG), out
        assert "bounded wait expired" in out[name], out
        assert out[name + "_after"], out
