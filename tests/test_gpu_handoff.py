"""Encoder -> decoder hand-off on the device (wg_job_upload_encoder_device).

A GPU encoder (internal/model/encoder.go:265-332 produces the [1500, d]
fp32 encoder output that Decode takes) can leave its output in device memory:
the job copies it device to device after waiting for the encoder's stream,
with no round trip through the host. The decode must be identical to the one
fed from host memory."""
import numpy as np
import pytest

import wgdec

pytestmark = pytest.mark.gpu
PROMPT = [50258, 50259, 50357, 50363]


@pytest.fixture(scope="module")
def model():
    m = wgdec.SyntheticModel(51864, 384, 6, 2, 448, "Q8_0", seed=19)
    dec = wgdec.WhisperDecoder(m)
    yield m, dec
    dec.close()
    m.close()


@pytest.mark.parametrize("beam", [1, 5])
def test_device_encoder_output_decodes_like_host(model, beam):
    torch = pytest.importorskip("torch")
    m, dec = model
    encs = [m.encoder_output(u) for u in range(3)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=beam, max_tokens=12, suppress_eot=True)
    ht, hl, hs = dec.decode_tokens(encs, params)
    # the "encoder" writes its outputs on a stream of its own
    s = torch.cuda.Stream(device="cuda:0")
    with torch.cuda.stream(s):
        dev = [torch.from_numpy(e).pin_memory().to("cuda:0", non_blocking=True) * 1.0 for e in encs]
    dt, dl, ds = dec.decode_tokens(dev, params, stream=s.cuda_stream)
    assert np.array_equal(ht, dt) and np.array_equal(hl, dl) and np.array_equal(hs, ds)


def test_device_upload_rejects_host_memory(model):
    m, dec = model
    enc = m.encoder_output(0, 64)
    job = wgdec.Job(dec, 1, 64, wgdec.DecoderParams(prompt=PROMPT, max_tokens=2))
    try:
        assert job.utterance_device(0) == 0
        with pytest.raises(wgdec.DecodeError) as ei:
            job.upload_device([enc.ctypes.data])
        assert ei.value.status == 1 and "device memory" in str(ei.value)
    finally:
        job.close()
