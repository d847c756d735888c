"""On-device top-k / top-p / temperature sampling (csrc/sample.cuh) against the oracle's restatement of the
session layer's sampler (oracle/xj_oracle.py:sample, ios/App/XJGlue.c:251-282) fed the same uniform draw
(SplitMix64 of seed and counter, oracle/xj_oracle.py:sample_uniform): the same id for every row, at the
LM head's width and a small vocabulary, several temperatures and top-p cuts; greedy at temperature 0;
equal logits at the k-th place taken lowest id first; sampled frequencies matching the sampler's
probabilities; and sampled decode through xj_cuda_decode equal to the reference CPU stage's logits
sampled on the host with the same draws."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import xj_oracle as xo

pytestmark = pytest.mark.gpu


def _rows(rng, rows, n, scale):
    return (rng.standard_normal((rows, n)) * scale).astype(np.float32)


@pytest.mark.parametrize("n,rows", [(151936, 8), (4096, 64), (300, 64), (40, 16), (17, 8)])
@pytest.mark.parametrize("temp", [0.3, 0.8, 1.5])
def test_sample_matches_host_sampler(n, rows, temp):
    from xjb200 import xjcuda
    rng = np.random.default_rng(n + int(temp * 10))
    lg = _rows(rng, rows, n, 3.0)
    seed, c0 = 1234567 + n, 77
    ids, mar = xjcuda.sample_logits(lg, temp, seed, c0)
    for r in range(rows):
        u = xo.sample_uniform(seed, c0 + r)
        want = xo.sample_fast(lg[r], temp, u) if n > 4096 else xo.sample(lg[r], temp, u)
        assert ids[r] == want, (r, ids[r], want)
        s = np.sort(lg[r])[::-1]
        assert mar[r] == pytest.approx(s[0] - s[1], abs=0)


@pytest.mark.parametrize("top_k,top_p", [(40, 0.95), (8, 0.5), (64, 1.0), (1, 0.95), (40, 0.05)])
def test_sample_top_k_top_p_settings(top_k, top_p):
    from xjb200 import xjcuda
    rng = np.random.default_rng(top_k)
    lg = _rows(rng, 48, 2048, 2.0)
    ids, _ = xjcuda.sample_logits(lg, 1.0, 99, 0, top_k=top_k, top_p=top_p)
    for r in range(48):
        want = xo.sample(lg[r], 1.0, xo.sample_uniform(99, r), top_k=top_k, top_p=top_p) if top_k > 1 else int(np.argmax(lg[r]))
        assert ids[r] == want, (r, top_k, top_p)


def test_temperature_zero_is_greedy_lowest_index():
    from xjb200 import xjcuda
    rng = np.random.default_rng(3)
    lg = _rows(rng, 16, 5000, 1.0)
    lg[3, [10, 20, 30]] = 9.0                       # ties: the lowest index wins
    ids, mar = xjcuda.sample_logits(lg, 0.0, 5)
    assert ids.tolist() == [int(np.argmax(r)) for r in lg]
    assert ids[3] == 10 and mar[3] == 0.0


def test_equal_logits_at_the_kth_place_take_lowest_ids():
    """3000 logits equal to the 40th largest value (more than the candidate buffer holds): the 35 larger
    ones plus the 5 lowest ids of the equal ones form the top-40 set."""
    from xjb200 import xjcuda
    rng = np.random.default_rng(4)
    n = 20000
    lg = (rng.standard_normal(n) * 0.1 - 5).astype(np.float32)
    big = rng.choice(n, 35, replace=False)
    lg[big] = 5 + np.arange(35, dtype=np.float32) * 0.01
    eq = np.setdiff1d(rng.choice(n, 3100, replace=False), big)[:3000]
    lg[eq] = 4.0
    allowed = set(big.tolist()) | set(np.sort(eq)[:5].tolist())
    ids, _ = xjcuda.sample_logits(np.tile(lg, (64, 1)), 50.0, 11, 0, top_k=40, top_p=1.0)
    assert set(ids.tolist()) <= allowed
    for r in range(64):
        assert ids[r] == xo.sample_fast(lg, 50.0, xo.sample_uniform(11, r), top_p=1.0)


def test_sampled_frequencies_follow_the_probabilities():
    """20000 draws from one 64-logit row at temperature 1 (top-40, top-p 0.95): chi-square against the
    sampler's own probabilities over the kept ids."""
    from xjb200 import xjcuda
    rng = np.random.default_rng(5)
    lg = (rng.standard_normal(64) * 1.5).astype(np.float32)
    N = 20000
    ids, _ = xjcuda.sample_logits(np.tile(lg, (N, 1)), 1.0, 2024, 0)
    order = np.lexsort((np.arange(64), -lg.astype(np.float64)))[:40]
    p = np.exp(lg[order].astype(np.float64) - lg[order[0]])
    cut = int(np.searchsorted(np.cumsum(p / p.sum()), 0.95) + 1)
    kept = order[:cut]
    pk = p[:cut] / p[:cut].sum()
    assert set(ids.tolist()) <= set(kept.tolist())
    cnt = np.array([(ids == k).sum() for k in kept], np.float64)
    chi2 = ((cnt - N * pk) ** 2 / (N * pk)).sum()
    assert chi2 < 3 * cut + 30, (chi2, cut)      # df = cut - 1; far beyond the 0.999 quantile only on a bug


@pytest.mark.parametrize("persist", [1, 0])
@pytest.mark.parametrize("which", ["tiny", "mid"])
def test_sampled_decode_matches_reference_stage(ref_lib, golden, tiny_path, mid_path, which, persist):
    """xj_cuda_decode with a sampler against the reference CPU stage's logits sampled on the host with the
    same draws (counter = position of the row that produced the logits), 24 tokens; then the same seed
    again, split over two calls, reproduces the ids. persist=1: the mid model samples inside the
    persistent kernel (its SAMPLE phase); the tiny model's F32 matrices keep it on the per-phase path."""
    from xjb200 import xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, persist)
    path = tiny_path if which == "tiny" else mid_path
    p = golden[f"{which}_prompt"]
    temp, seed, n_gen = 0.9, 424242, 24
    rm = ref_lib.Model(path)
    rs = ref_lib.Stage(rm, 0, rm.n_layer, 256, 8)
    lg = None
    for i in range(0, len(p), 8):
        x = rs.forward(rm.embed_many(p[i:i + 8]))
        lg = rs.logits(x[-1:])[0]
    want = []
    for g in range(n_gen):
        t = xo.sample(lg, temp, xo.sample_uniform(seed, len(p) - 1 + g))
        want.append(t)
        if g + 1 < n_gen:
            lg = rs.logits(rs.forward(rm.embed_many([t])))[0]
    rs.close()
    rm.close()
    m = xjcuda.Model(path)
    s = xjcuda.Stage(m, 0, m.n_layer, 256, 8)
    s.set_sampler(temp, seed)
    toks, _, _ = s.decode(p, n_gen)
    assert toks.tolist() == want
    if which == "mid":
        assert s.last_decode_launches()[1] == (1 if persist else (n_gen - 1) * xjcuda.lib().xj_cuda_graph_kernels(s.addr))
    s.reset()
    a, _, _ = s.decode(p, 10)                  # ids 0..9; id 9 is emitted, not yet fed
    b, _, _ = s.decode(a[-1:], n_gen - 10)     # feeds id 9, emits ids 10..23
    assert a.tolist() + b.tolist() == want
    s.set_sampler(0.0)
    s.reset()
    g0, _, _ = s.decode(p, 8)
    assert g0.tolist() == golden[f"{which}_tokens"][:8].tolist()
    s.close()
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)
