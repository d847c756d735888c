"""Batched decode of independent sequences (xj_cuda_batch_*) against single-sequence decode.

Every matrix-vector product computes each token's column independently in a fixed order, and the
attention / Gated-DeltaNet / greedy-pick kernels of the batch run the single-sequence device code on
each sequence's own state. Up to 16 sequences the matrix-vector kernels are the single-sequence
arithmetic, so sequence b of a batch must produce exactly (bit for bit, margins included) what
xj_cuda_decode produces for that sequence alone; above 16 the 64-token kernel adds K in another order
(fp32-level differences), so the ids must still agree and the margins to fp32 accuracy. One of the
sequences is the golden prompt, whose ids are the reference's.
"""
from __future__ import annotations

import numpy as np
import pytest

from make_golden import C0_N_GEN, MID_N_GEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xc():
    from xjb200 import xjcuda
    xjcuda.lib()
    yield xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)
    xjcuda.set_option(xjcuda.OPT_KV_F32, 0)


def prompts_with_golden(golden, which, n_seq, vocab):
    p0 = golden[f"{which}_prompt"]
    rng = np.random.default_rng(11)
    rest = rng.integers(0, vocab, (n_seq - 1, len(p0))).astype(np.int32)
    return np.concatenate([p0[None, :], rest], axis=0)


def single(xc, m, prompt, n_gen):
    xc.set_option(xc.OPT_PERSIST, 0)
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    out = s.decode(prompt, n_gen, want_margins=True)
    s.close()
    return out


@pytest.mark.parametrize("which,n_seq", [("config0", 1), ("config0", 5), ("mid", 3), ("config0", 24), ("mid", 20),
                                         ("mid", 64)])
def test_batch_matches_single_sequence_decode(xc, golden, config0_path, mid_path, which, n_seq):
    xc.set_option(xc.OPT_KV_F32, 0)
    m = xc.Model(config0_path if which == "config0" else mid_path)
    n_gen = C0_N_GEN if which == "config0" else MID_N_GEN
    P = prompts_with_golden(golden, which, n_seq, m.n_vocab)
    b = xc.Batch(m, n_seq, 512)
    toks, mar, ms = b.decode(P, n_gen, want_margins=True)
    assert toks[0].tolist() == golden[f"{which}_tokens"].tolist()
    assert b.n_past == P.shape[1] + n_gen - 1 and ms[1] > 0
    for i in range(min(n_seq, 3)):
        t1, m1, _ = single(xc, m, P[i], n_gen)
        assert toks[i].tolist() == t1.tolist(), i
        if n_seq <= 16:
            assert np.array_equal(mar[i], m1), i
        else:
            assert np.allclose(mar[i], m1, rtol=1e-2, atol=5e-4), (i, np.abs(mar[i] - m1).max())
    pre, dec = b.last_launches()
    assert pre > 0 and dec > 0
    b.close()


def test_batch_continuation_reset_and_fp32_kv(xc, golden, mid_path):
    """Two calls continue the sequences; reset starts over; the fp32 KV cache gives the reference ids."""
    xc.set_option(xc.OPT_KV_F32, 1)
    m = xc.Model(mid_path)
    P = prompts_with_golden(golden, "mid", 4, m.n_vocab)
    b = xc.Batch(m, 4, 512)
    xc.set_option(xc.OPT_KV_F32, 0)
    full, _, _ = b.decode(P, 30)
    b.reset()
    a, _, _ = b.decode(P, 12)
    c, _, _ = b.decode(a[:, -1:], 18)     # the last id of each sequence was not fed back: feed it now
    assert np.array_equal(np.concatenate([a, c], axis=1), full)
    assert full[0].tolist() == golden["mid_tokens"][:30].tolist()
    b.close()


def test_batch_errors(xc, config0_path):
    m = xc.Model(config0_path)
    b = xc.Batch(m, 2, 40)
    with pytest.raises(xc.XjError):
        b.decode(np.zeros((2, 30), np.int32), 20)          # 30 + 20 - 1 > 40
    with pytest.raises(xc.XjError):
        xc.Batch(m, 0, 40)
    b.close()
