"""The persistent step kernel (WG_STEP_KERNEL=1, opt-in): every layer of a
token step of a small batch in one cooperative launch. Run in child
processes (the switch is read when a job is created): teacher-forced logits
within the decoder's gates at a d=384 and a large-v3-width model, in both
modes, and a beam-5 decode that runs to its length."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
import wgdec

pytestmark = pytest.mark.gpu
PROMPT = [50258, 50259, 50357, 50363]

_SCRIPT = r"""
import sys, json, numpy as np
sys.path[:0] = [{pkg!r}]
import wgdec
m = wgdec.SyntheticModel({V}, {d}, {d} // 64, {L}, 448, {qt!r}, seed=5)
dec = wgdec.WhisperDecoder(m)
encs = [m.encoder_output(u, 300) for u in range({U})]
forced = np.random.default_rng(4).integers(0, 50257, size=({U}, {n}))
out = dict(mode={mode})
out["logits"] = dec.teacher_forced_logits(encs, [50258, 50259, 50357, 50363], forced, {mode}).tolist()
params = wgdec.DecoderParams(prompt=[50258, 50259, 50357, 50363], beam_size=5, max_tokens=12, mode={mode},
                             suppress_eot=True)
t, l, s = dec.decode_tokens(encs, params)
out["tokens"] = t.tolist(); out["lens"] = l.tolist()
j = wgdec.Job(dec, {U}, 300, params)
j.upload(encs)
out["uses_step"] = j.uses_step_kernel()
j.close()
print(json.dumps(out))
"""


def _run(step, **kw):
    code = _SCRIPT.format(pkg=str(wgdec.PKG), **kw)
    env = dict(os.environ, WG_STEP_KERNEL="1" if step else "0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("V,d,L,qt,U,n,mode", [(51864, 384, 2, "Q8_0", 3, 6, wgdec.MODE_CORRECT),
                                               (51864, 384, 2, "Q5_1", 1, 6, wgdec.MODE_REF_COMPAT),
                                               (51866, 1280, 2, "Q8_0", 1, 4, wgdec.MODE_CORRECT)])
def test_step_kernel_matches_the_oracle_and_the_kernel_chain(V, d, L, qt, U, n, mode):
    kw = dict(V=V, d=d, L=L, qt=qt, U=U, n=n, mode=mode)
    on, off = _run(True, **kw), _run(False, **kw)
    assert on["uses_step"] and not off["uses_step"]
    lg = np.asarray(on["logits"], dtype=np.float32)
    m = wgdec.SyntheticModel(V, d, d // 64, L, 448, qt, seed=5)
    encs = [m.encoder_output(u, 300) for u in range(U)]
    forced = np.random.default_rng(4).integers(0, 50257, size=(U, n))
    for u in range(U):
        ref = oracle.teacher_forced(m, encs[u], PROMPT, forced[u], mode, V)
        for s in range(n):
            err = float(np.max(np.abs(lg[s, u] - ref[s])))
            assert err <= 2e-2 and err <= 1e-3 * float(np.max(np.abs(ref[s]))), (u, s, err)
    m.close()
    # and the decode itself runs on it (token ids in range, every row stepped)
    toks = np.asarray(on["tokens"])
    assert (toks >= 0).all() and (toks < V).all() and all(l == len(PROMPT) + 12 for l in on["lens"])
