"""Greedy speculative decoding with a separate draft model (xj_cuda_spec_decode, config 4).

The reference invariant (e2e.sh: speculative output equals plain greedy) is checked against the
reference's own ids for the golden prompt (oracle) and against plain device decode through the same
kernels: with the target model itself as the draft every drafted token is accepted (the accept-all path
and its bonus pick), with an unrelated small draft almost none is (the reject path: rollback of the
target through its checkpoints, restore and re-feed of the draft)."""
from __future__ import annotations

import numpy as np
import pytest

from make_golden import MID_N_GEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xc():
    from xjb200 import xjcuda
    xjcuda.lib()
    yield xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)


def plain(xc, m, prompt, n_gen):
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    toks, _, _ = s.decode(prompt, n_gen)
    s.close()
    return toks


@pytest.mark.parametrize("k", [1, 4])
@pytest.mark.parametrize("draft_kind", ["self", "small"])
def test_speculative_equals_plain_greedy(xc, golden, mid_path, mid_draft_path, k, draft_kind):
    xc.set_option(xc.OPT_PERSIST, 0)
    m = xc.Model(mid_path)
    dm = m if draft_kind == "self" else xc.Model(mid_draft_path)
    p = golden["mid_prompt"]
    want = golden["mid_tokens"]
    assert plain(xc, m, p, MID_N_GEN).tolist() == want.tolist()
    t = xc.Stage(m, 0, m.n_layer, 512, 8)
    d = xc.Stage(dm, 0, dm.n_layer, 512, 8)
    toks, (rounds, drafted, accepted, refeeds) = t.spec_decode(d, p, MID_N_GEN, k)
    assert toks.tolist() == want.tolist()
    assert t.s.n_past == len(p) + MID_N_GEN - 1 and d.s.n_past == len(p) + MID_N_GEN - 1
    assert rounds >= 1 and 0 <= accepted <= drafted
    if draft_kind == "self":
        assert accepted == drafted and rounds <= (MID_N_GEN - 1 + k) // (k + 1) + 1
    # a second call continues from the stages' positions like plain decode does
    more, _ = t.spec_decode(d, toks[-1:], 8, k)
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    ref = s.decode(np.concatenate([p, toks[:-1]]), 1)[0]
    ref2 = s.decode(toks[-1:], 8)[0]
    assert more.tolist() == ref2.tolist()
    for x in (t, d, s):
        x.close()


def test_speculative_errors(xc, mid_path, config0_path):
    m = xc.Model(mid_path)
    other = xc.Model(config0_path)                      # another vocabulary
    t = xc.Stage(m, 0, m.n_layer, 256, 8)
    d = xc.Stage(other, 0, other.n_layer, 256, 8)
    with pytest.raises(xc.XjError):
        t.spec_decode(d, np.array([1, 2, 3], np.int32), 4, 4)
    d2 = xc.Stage(m, 0, m.n_layer, 256, 8)
    with pytest.raises(xc.XjError):
        t.spec_decode(d2, np.array([1, 2, 3], np.int32), 4, 8)   # k + 1 > max_batch
    with pytest.raises(xc.XjError):
        t.spec_decode(t, np.array([1, 2, 3], np.int32), 4, 2)    # the draft is the target stage
    for x in (t, d, d2):
        x.close()



# ---- batched speculative decoding (xj_cuda_batch_spec_decode): every sequence of a batch at once
@pytest.mark.parametrize("n_seq", [3, 20])
@pytest.mark.parametrize("own_draft", [True, False])
def test_batch_spec_decode_equals_plain_greedy(mid_path, mid_draft_path, n_seq, own_draft):
    """Batched verify of k + 1 = 5 tokens per sequence: 3 sequences (15 verify rows, the wide kernel) and
    20 (100 rows, the tcgen05 kernel; chunked prompts) against plain batch decoding; with the target as its
    own draft every drafted token is accepted, with the small draft nearly none."""
    from xjb200 import xjcuda
    rng = np.random.default_rng(n_seq)
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (n_seq, 12)).astype(np.int32)
    n_gen, k = 24, 4
    b = xjcuda.Batch(m, n_seq, 256)
    want, _, _ = b.decode(prompts, n_gen)
    b.close()
    dm = m if own_draft else xjcuda.Model(mid_draft_path)
    target = xjcuda.Batch(m, n_seq, 256, max_tokens=k + 1)
    draft = xjcuda.Batch(dm, n_seq, 256, max_tokens=4)
    got, st, ms = target.spec_decode(draft, prompts, n_gen, k)
    target.close()
    draft.close()
    assert np.array_equal(got, want)
    rounds, drafted, accepted, rows = st
    assert drafted == rounds * k * n_seq and rows == rounds * (k + 1) and ms > 0
    if own_draft:
        assert accepted == drafted and rounds == -(-(n_gen - 1) // (k + 1))
    else:
        assert rounds <= n_gen - 1


def test_batch_chunked_prompt_equals_token_by_token(mid_path):
    """A batch of 20 sequences taking its prompts in chunks of 8 tokens per sequence gives the ids and
    margins of the one-token steps, bit for bit."""
    from xjb200 import xjcuda
    rng = np.random.default_rng(5)
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (20, 21)).astype(np.int32)
    a = xjcuda.Batch(m, 20, 256)
    ia, ma, _ = a.decode(prompts, 8, want_margins=True)
    a.close()
    c = xjcuda.Batch(m, 20, 256, max_tokens=8)
    ic, mc, _ = c.decode(prompts, 8, want_margins=True)
    c.close()
    assert np.array_equal(ia, ic)
    assert ma.view(np.uint32).tolist() == mc.view(np.uint32).tolist()
