"""The token-selection kernels on given logits (wg_sample_test) against the
oracle's restatement of the reference's samplers, at the row counts where
each variant runs: up to 64 rows a row is split over an 8-CTA cluster, above
64 one CTA takes a row (the benchmark's 320 rows).

* greedy (sampleGreedyWithScratch, decoder.go:996-1059): identical tokens,
  including exact ties (the first maximum wins) and the SuppressNST re-pick;
* top-5 (topKTokensWithScratch, :1068-1136): identical tokens and order,
  including exact ties (replace-min scan order), log-probs within 3e-5 (the
  float32 sum of 51,866 exponentials in another order moves log Z by ~1e-5);
* the top-p fallback (:1036-1056, :1251-1378) with the seeded draw
  wg_uniform(seed, row, step): identical tokens except where the draw or the
  0.9 nucleus boundary falls within 5e-5 of a cumulative-probability
  boundary. The GPU sums the probabilities exactly in fixed point; the
  reference sums them in float32 in sorted order, whose rounding (~1e-5
  after tens of thousands of terms) is itself as large as one token's
  probability in a flat distribution, so there a pick one place away is the
  reference arithmetic's own uncertainty.

The repetition penalty (decoder.go:1140-1167) is applied by these kernels to
every row from its history first, as in the decode."""
import numpy as np
import pytest

import oracle
import wgdec

pytestmark = pytest.mark.gpu
V, EOT = 51866, 50256


def rows(R, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal((R, V)) * scale).astype(np.float32)
    hist = rng.integers(0, V, size=(R, 40)).astype(np.int32)
    hist[:, :5] = np.argmax(lg[:, :], axis=1)[:, None]  # the favourite was said five times: penalty 10
    return lg, hist


def penalised(lg, hist):
    return np.stack([oracle.apply_penalty(lg[r], hist[r]) for r in range(lg.shape[0])])


@pytest.mark.parametrize("R", [40, 80])
def test_greedy_kernels(R):
    lg, hist = rows(R, R)
    # exact ties of the row maximum at a later index on some rows (first one wins)
    for r in range(0, R, 7):
        j = int(np.argmax(lg[r]))
        lg[r, (j + 1000) % V] = lg[r, j]
        hist[r, :5] = 0
    params = wgdec.DecoderParams(prompt=[0], beam_size=1)
    got = wgdec.sample(lg, hist, EOT, params)
    pen = penalised(lg, hist)
    want = [oracle.sample_greedy(pen[r], EOT, 1.0) for r in range(R)]
    assert got.tolist() == want


@pytest.mark.parametrize("R", [40, 80])
def test_greedy_suppress_nst(R):
    lg, hist = rows(R, 100 + R)
    hist[:, :5] = 1
    pen = penalised(lg, hist)
    eot = int(np.argmax(pen[0]))  # row 0's best token is "EOT"
    thold = float(-pen[0, eot]) - 0.25  # logits[eot] < -thold on row 0: re-pick
    params = wgdec.DecoderParams(prompt=[0], beam_size=1, suppress_nst=True, no_speech_thold=thold)
    got = wgdec.sample(lg, hist, eot, params)
    want = [oracle.sample_greedy(pen[r], eot, 1.0, True, thold) for r in range(R)]
    assert got.tolist() == want and got[0] != eot


@pytest.mark.parametrize("R", [40, 80])
@pytest.mark.parametrize("temperature", [0.0, 0.7])
def test_topk_kernels(R, temperature):
    lg, hist = rows(R, 200 + R)
    for r in range(0, R, 5):  # exact ties inside and at the edge of the top 5
        order = np.argsort(-lg[r], kind="stable")
        lg[r, order[6]] = lg[r, order[3]]
        lg[r, order[2]] = lg[r, order[1]]
    params = wgdec.DecoderParams(prompt=[0], beam_size=5, temperature=temperature)
    tok, lp = wgdec.sample(lg, hist, EOT, params)
    pen = penalised(lg, hist)
    for r in range(R):
        wt, wl = oracle.topk(pen[r], 5, temperature if temperature > 0 else 1.0)
        assert tok[r].tolist() == wt.tolist(), r
        np.testing.assert_allclose(lp[r], wl, atol=3e-5, rtol=0)


def uniform_py(seed, u, t):
    """wg_uniform restated in Python (checks the oracle's copy of the header function)."""
    M = 0xFFFFFFFFFFFFFFFF
    z = (seed ^ ((u + 1) * 0x9E3779B97F4A7C15 & M) ^ ((t + 1) * 0xD1B54A32D192ED03 & M)) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    z ^= z >> 31
    return np.float32(z >> 40) * np.float32(1.0 / 16777216.0)


def test_uniform_contract():
    for seed, u, t in [(0, 0, 0), (1, 2, 3), (2 ** 63 + 5, 63, 447), (12345, 7, 100)]:
        assert uniform_py(seed, u, t) == np.float32(oracle.uniform(seed, u, t))
        assert 0.0 <= oracle.uniform(seed, u, t) < 1.0


def reference_walk(pen_row, temperature, u01):
    """The reference's nucleus order, cumulative float32 mass, cut and draw;
    returns (order, cum, k_star, r) for the ambiguity checks."""
    it = np.float32(1.0 / temperature)
    sc = (pen_row * it).astype(np.float32)
    m = sc.max()
    es = np.float32(0)
    for v in np.exp((sc - m).astype(np.float64)).astype(np.float32):
        es = np.float32(es + v)
    logz = np.float32(np.float32(np.log(np.float64(es))) + m)
    p = np.exp((sc - logz).astype(np.float64)).astype(np.float32)
    order = np.lexsort((np.arange(sc.size), -sc))
    cum = np.cumsum(p[order], dtype=np.float32)
    k = int(np.searchsorted(cum >= np.float32(0.9), True))  # first index with cum >= 0.9
    k = min(k, cum.size - 1)
    r = np.float32(np.float32(u01) * cum[k])
    return order, cum, k, r


@pytest.mark.parametrize("R", [40, 80])
@pytest.mark.parametrize("temperature", [1.0, 1.4])
def test_topp_fallback_kernel(R, temperature):
    # rows from flat (scale 0.5: thousands of tokens in the nucleus) to peaky
    # (scale 6: the first few); LogprobThold 3 sends the flat ones to top-p
    scales = np.linspace(0.5, 6.0, R).astype(np.float32)
    lg, hist = rows(R, 300 + R)
    lg *= scales[:, None]
    seed, step = 424242, 17
    params = wgdec.DecoderParams(prompt=[0], beam_size=1, temperature=temperature, logprob_thold=3.0, seed=seed)
    got = wgdec.sample(lg, hist, EOT, params, step=step)
    pen = penalised(lg, hist)
    exact = ambiguous = fallback = 0
    for r in range(R):
        g = oracle.sample_greedy(pen[r], EOT, temperature)
        if not oracle.topp_fallback(pen[r], g, temperature, 3.0):
            assert got[r] == g, r
            exact += 1
            continue
        fallback += 1
        u01 = oracle.uniform(seed, r, step)
        want = oracle.sample_topp(pen[r], temperature, u01)
        if got[r] == want:
            exact += 1
            continue
        order, cum, k, rr = reference_walk(pen[r], temperature, u01)
        pos_g, pos_w = int(np.nonzero(order == got[r])[0][0]), int(np.nonzero(order == want)[0][0])
        near_cut = min(abs(cum[k] - 0.9), abs(cum[k - 1] - 0.9) if k else 1.0) <= 5e-5
        lo, hi = min(pos_g, pos_w), max(pos_g, pos_w)
        near_draw = np.all(np.abs(cum[lo:hi] - rr) <= 5e-5)
        assert near_cut or near_draw, (r, pos_g, pos_w, float(rr), cum[lo:hi + 1])
        ambiguous += 1
    assert fallback >= R // 4 and exact >= R * 4 // 5, (exact, ambiguous, fallback)
