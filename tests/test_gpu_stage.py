"""Parity of the CUDA stage (libxj_cuda.so, called through its C ABI) with the reference CPU path.

Gates (north star): dequantised blocks bit-exact; per-layer activations and logits within 1e-2
relative error (fp32 accumulate; 1e-4 with the fp32 KV cache); greedy tokens identical for 64 steps.
The expected values are the committed golden outputs of the reference (tests/golden/make_golden.py)
and, where the reference library is present, the reference run live in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err
from make_golden import C0_N_GEN, DQ_K, DQ_ROWS, MID_N_GEN, TINY_N_GEN, TRACE_CHUNKS
from oracle import xj_oracle as xo

pytestmark = pytest.mark.gpu

TYPES = (xo.F16, xo.BF16, xo.Q8_0, xo.Q4_K, xo.Q5_K, xo.Q6_K)


@pytest.fixture(scope="module")
def xc():
    from xjb200 import xjcuda
    xjcuda.lib()
    yield xjcuda
    xjcuda.set_option(xjcuda.OPT_KV_F32, 0)
    xjcuda.set_option(xjcuda.OPT_GEMV, 0)
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)


def model_path(which, tiny_path, config0_path, mid_path=None):
    return {"tiny": tiny_path, "config0": config0_path, "mid": mid_path}[which]


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact(xc, golden, t):
    got = xc.dequant_rows(t, golden[f"dq_{t}_raw"].tobytes(), DQ_K, DQ_ROWS)
    assert got.view(np.uint32).tolist() == golden[f"dq_{t}_f32"].view(np.uint32).tolist()


@pytest.mark.parametrize("which", ["tiny", "config0"])
@pytest.mark.parametrize("kv32,gemv", [(0, 0), (1, 0), (1, 1)])
def test_layer_trace(xc, golden, tiny_path, config0_path, which, kv32, gemv):
    xc.set_option(xc.OPT_KV_F32, kv32)
    xc.set_option(xc.OPT_GEMV, gemv)
    m = xc.Model(model_path(which, tiny_path, config0_path))
    L = m.n_layer
    stages = [xc.Stage(m, l, l + 1, 128, 16, has_head=(l == L - 1)) for l in range(L)]
    p = golden[f"{which}_prompt"]
    want_hid, want_lg = golden[f"{which}_trace_hid"], golden[f"{which}_trace_logits"]
    tol = 1e-4 if kv32 else 1e-2
    pos = 0
    for c, T in enumerate(TRACE_CHUNKS):
        x = m.embed_many(p[pos:pos + T])
        for l, s in enumerate(stages):
            x = s.forward(x)
            if c == len(TRACE_CHUNKS) - 1:
                assert rel_err(x, want_hid[l + 1]) < tol, (which, l, rel_err(x, want_hid[l + 1]))
        pos += T
    assert rel_err(stages[-1].logits(x), want_lg) < tol
    assert np.argmax(stages[-1].logits(x)[-1]) == np.argmax(want_lg[-1])


@pytest.mark.parametrize("which", ["tiny", "config0"])
@pytest.mark.parametrize("kv32", [0, 1])
def test_greedy_tokens_identical_vtable(xc, golden, tiny_path, config0_path, which, kv32):
    """64 (48 for the tiny model) greedy steps through forward/logits with host buffers."""
    xc.set_option(xc.OPT_KV_F32, kv32)
    m = xc.Model(model_path(which, tiny_path, config0_path))
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    p = golden[f"{which}_prompt"]
    n_gen = TINY_N_GEN if which == "tiny" else C0_N_GEN
    lg = None
    for i in range(0, len(p), 8):
        x = s.forward(m.embed_many(p[i:i + 8]))
        lg = s.logits(x[-1:])[0]
    toks = []
    for g in range(n_gen):
        t = int(np.argmax(lg))
        toks.append(t)
        if g + 1 < n_gen:
            lg = s.logits(s.forward(m.embed(t)[None, :]))[0]
    assert toks == golden[f"{which}_tokens"].tolist()
    assert s.n_past == len(p) + n_gen - 1


@pytest.mark.parametrize("persist", [0, 1])
@pytest.mark.parametrize("which", ["tiny", "config0", "mid"])
def test_greedy_tokens_identical_device_decode(xc, golden, tiny_path, config0_path, mid_path, which, persist):
    """xj_cuda_decode against the reference's greedy tokens, through the per-step graph (persist=0) and
    the persistent kernel (persist=1; the tiny model's F32 matrices keep it on the graph path)."""
    xc.set_option(xc.OPT_KV_F32, 0)
    xc.set_option(xc.OPT_GEMV, 0)
    xc.set_option(xc.OPT_PERSIST, persist)
    m = xc.Model(model_path(which, tiny_path, config0_path, mid_path))
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    p = golden[f"{which}_prompt"]
    n_gen = {"tiny": TINY_N_GEN, "config0": C0_N_GEN, "mid": MID_N_GEN}[which]
    toks, margins, ms = s.decode(p, n_gen, want_margins=True)
    assert toks.tolist() == golden[f"{which}_tokens"].tolist()
    assert np.allclose(margins, golden[f"{which}_margins"], rtol=0.05, atol=2e-3)
    assert s.n_past == len(p) + n_gen - 1 and ms[1] > 0
    pre, launches = s.last_decode_launches()
    assert pre > 0
    if persist and which != "tiny":
        assert launches == 1
    else:
        assert launches == (n_gen - 1) * xc.lib().xj_cuda_graph_kernels(s.addr) > n_gen
    # a second call continues the same sequence; reset starts over and reproduces the first call
    s.reset()
    toks2, _, _ = s.decode(p, n_gen)
    assert toks2.tolist() == toks.tolist()


@pytest.mark.parametrize("which", ["config0", "mid"])
def test_persistent_decode_kv_f32_and_continuation(xc, golden, config0_path, mid_path, which):
    """The persistent kernel with the fp32 KV cache, and a decode split into two calls (the second call
    continues from the first one's position and state) against the reference's tokens."""
    xc.set_option(xc.OPT_PERSIST, 1)
    xc.set_option(xc.OPT_GEMV, 0)
    xc.set_option(xc.OPT_KV_F32, 1)
    m = xc.Model(model_path(which, None, config0_path, mid_path))
    s = xc.Stage(m, 0, m.n_layer, 512, 8)
    xc.set_option(xc.OPT_KV_F32, 0)
    p = golden[f"{which}_prompt"]
    want = golden[f"{which}_tokens"].tolist()
    a, _, _ = s.decode(p, 20)
    assert s.last_decode_launches()[1] == 1
    # the last emitted id is not fed back: passing it as a one-token prompt continues the sequence
    b, _, _ = s.decode(a[-1:], len(want) - 20)
    assert a.tolist() + b.tolist() == want


def test_persistent_matches_graph_path_long_context(xc, mid_path):
    """Long run (attention over up to ~1000 positions, split across CTAs) through both CUDA paths: the
    ids agree until the first step whose top-2 gap is a near tie (the two paths sum GDN and attention
    in different orders)."""
    xc.set_option(xc.OPT_GEMV, 0)
    xc.set_option(xc.OPT_KV_F32, 0)
    m = xc.Model(mid_path)
    p = np.random.default_rng(5).integers(0, m.n_vocab, 700).astype(np.int32)
    out = {}
    for persist in (0, 1):
        xc.set_option(xc.OPT_PERSIST, persist)
        s = xc.Stage(m, 0, m.n_layer, 1100, 64)
        out[persist] = s.decode(p, 300, want_margins=True)
        assert s.last_decode_launches()[1] == (1 if persist else 299 * xc.lib().xj_cuda_graph_kernels(s.addr))
        s.close()
    (t0, m0, _), (t1, m1, _) = out[0], out[1]
    diff = np.nonzero(t0 != t1)[0]
    first = int(diff[0]) if diff.size else len(t0)
    assert first >= 100 or m0[first] < 5e-3, (first, m0[first])
    assert np.allclose(m0[:first], m1[:first], rtol=0.05, atol=2e-3)


def test_persistent_attention_several_rounds_per_split(xc, mid_path, ref_lib):
    """Context longer than the persistent kernel's splits hold in one round (mid: 2 KV heads, 74 splits of
    32 positions = 2368): every attention item walks several rounds of cached rows and the new row
    enters in a later round. The ids must equal the reference's CPU path until a near tie."""
    xc.set_option(xc.OPT_GEMV, 0)
    xc.set_option(xc.OPT_KV_F32, 0)
    xc.set_option(xc.OPT_PERSIST, 1)
    m = xc.Model(mid_path)
    p = np.random.default_rng(21).integers(0, m.n_vocab, 2600).astype(np.int32)
    s = xc.Stage(m, 0, m.n_layer, 2700, 64)
    toks, mar, _ = s.decode(p, 40, want_margins=True)
    assert s.last_decode_launches()[1] == 1
    s.close()
    rm = ref_lib.Model(mid_path)
    want, want_mar, _, _ = rm.greedy(p, 40, max_batch=64, n_ctx=2700)
    rm.close()
    diff = np.nonzero(toks != want)[0]
    first = int(diff[0]) if diff.size else len(toks)
    assert first >= 20 or want_mar[first] < 5e-3, (first, want_mar[first])
    assert np.allclose(mar[:first], want_mar[:first], rtol=0.05, atol=2e-3)


def test_reference_driver_runs_cuda_stage(xc, ref_lib, golden, tiny_path, config0_path):
    """The reference's own loader builds the xj_model and its greedy loop drives the CUDA stage."""
    for which in ("tiny", "config0"):
        rm = ref_lib.Model(model_path(which, tiny_path, config0_path))
        n_gen = TINY_N_GEN if which == "tiny" else C0_N_GEN
        toks, mar, first, _ = rm.greedy(golden[f"{which}_prompt"], n_gen, max_batch=8, n_ctx=512, ctor=xc.ctor_address())
        assert toks.tolist() == golden[f"{which}_tokens"].tolist()
        assert rel_err(first, golden[f"{which}_first_logits"]) < 1e-2


@pytest.mark.parametrize("k", [0, 1, 3, 4])
def test_speculative_loop_through_reference_pipeline(xc, ref_lib, golden, tiny_path, k):
    """The reference pipeline + MTP speculative loop (core/xj_spec.c) with CUDA stages for the trunk and
    the MTP head: output identical to plain greedy (tests/e2e.sh:70-103 invariant)."""
    rm = ref_lib.Model(tiny_path)
    toks, stats = rm.spec(golden["tiny_prompt"], TINY_N_GEN, k, max_batch=8, n_ctx=512, ctor=xc.ctor_address())
    assert toks.tolist() == golden["tiny_tokens"].tolist()
    # oracle drafts with planted misses exercise accept-all / accept-some / rollback paths
    toks, stats = rm.spec(golden["tiny_prompt"], TINY_N_GEN, k, max_batch=8, n_ctx=512, ctor=xc.ctor_address(),
                          oracle=golden["tiny_tokens"], oracle_miss=3)
    assert toks.tolist() == golden["tiny_tokens"].tolist()
    if k:
        assert stats[2] > 0


def test_split_pipeline_through_reference(xc, ref_lib, golden, tiny_path):
    rm = ref_lib.Model(tiny_path)
    toks, _ = rm.spec(golden["tiny_prompt"], TINY_N_GEN, 0, max_batch=8, n_ctx=512, s1=3, ctor=xc.ctor_address())
    assert toks.tolist() == golden["tiny_split3"].tolist()


def test_rollback_equivalence(xc, tiny_path, config0_path):
    """tools/xjpipe-check.c:78-109 on the CUDA stage: forward 6, forward 4 with keep, roll back to 8,
    forward 2 new == a fresh run over the same tokens."""
    for path in (tiny_path, config0_path):
        m = xc.Model(path)
        toks = np.random.default_rng(11).integers(0, m.n_vocab, 16)
        s = xc.Stage(m, 0, m.n_layer, 64, 16)
        s.forward(m.embed_many(toks[:6]))
        s.keep = 4
        s.forward(m.embed_many(toks[6:10]))
        assert s.ck == (6, 4) and s.keep == 0
        s.rollback(8)
        out = s.forward(m.embed_many(toks[12:14]))
        f = xc.Stage(m, 0, m.n_layer, 64, 16)
        want = f.forward(m.embed_many(np.concatenate([toks[:8], toks[12:14]])))[-2:]
        assert rel_err(out, want) < 1e-5
        with pytest.raises(xc.XjError):
            s.rollback(3)


def test_mtp_stage_matches_oracle(xc, tiny_path):
    """MTP stage (l0 = n_layer): [embedding | hidden] -> eh_proj -> MTP layer, then shared_head_norm + head."""
    m = xc.Model(tiny_path)
    om = xo.Model(tiny_path)
    L, E = m.n_layer, m.n_embd
    s = xc.Stage(m, L, L + 1, 64, 8)
    os_ = xo.Stage(om, L, L + 1, 64, 8)
    assert s.s.mtp
    rng = np.random.default_rng(5)
    for T in (3, 1):
        x = np.concatenate([m.embed_many(rng.integers(0, m.n_vocab, T)),
                            rng.standard_normal((T, E)).astype(np.float32) * 3], axis=1)
        h, oh = s.forward(x), os_.forward(x)
        assert rel_err(h, oh) < 1e-2
        assert rel_err(s.logits(h), os_.logits(oh)) < 1e-2


def test_errors(xc, tiny_path):
    m = xc.Model(tiny_path)
    s = xc.Stage(m, 0, 2, 8, 4, has_head=False)
    with pytest.raises(xc.XjError):
        s.forward(np.zeros((5, m.n_embd), np.float32))           # T > max_batch
    s.keep = 3
    with pytest.raises(xc.XjError):
        s.forward(np.zeros((5, m.n_embd), np.float32))
    assert s.keep == 0                                            # keep is cleared on failure too
    s.forward(np.zeros((4, m.n_embd), np.float32))
    s.forward(np.zeros((4, m.n_embd), np.float32))
    with pytest.raises(xc.XjError, match="full"):
        s.forward(np.zeros((1, m.n_embd), np.float32))           # n_past + T > n_ctx
    with pytest.raises(xc.XjError):
        s.logits(np.zeros((1, m.n_embd), np.float32))            # no head
    with pytest.raises(xc.XjError):
        xc.Stage(m, 3, 2)                                         # bad layer range
    with pytest.raises(xc.XjError):
        xc.Stage(m, 0, m.n_layer + 2)
