"""Models whose matrices are Q5_K, F16 or BF16 (the reference decodes them in core/xj_quant.h:55-122)
stay on the tensor-core paths: the persistent decode kernel, the 1..4-token and 5..16-token GEMVs, and
batches wider than 16 rows in 16-token chunks. Greedy tokens must equal the reference's own CPU path
(oracle/_ref, core/*.c) on the same synthetic model, with the top-2 margins close."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import xj_oracle as xo

pytestmark = pytest.mark.gpu

N_PROMPT, N_GEN = 24, 24


@pytest.fixture(scope="module")
def xc():
    from xjb200 import xjcuda
    xjcuda.lib()
    yield xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)


@pytest.fixture(scope="module", params=[xo.Q5_K, xo.F16, xo.BF16], ids=["q5_k", "f16", "bf16"])
def typed_model(request, tmp_path_factory, ref_lib):
    from xjb200 import synth
    cfg = synth.MID.replace(name=f"mid-w{request.param}", wtype=request.param)
    path = synth.cached_gguf(cfg, tmp_path_factory.mktemp("typed"))
    p = np.random.default_rng(request.param).integers(0, cfg.n_vocab, N_PROMPT).astype(np.int32)
    rm = ref_lib.Model(path)
    tok, mar, _, _ = rm.greedy(p, N_GEN, max_batch=8, n_ctx=256)
    rm.close()
    return request.param, path, p, tok, mar


@pytest.mark.parametrize("persist", [1, 0])
def test_typed_model_greedy_matches_reference(xc, typed_model, persist):
    t, path, p, want, want_mar = typed_model
    xc.set_option(xc.OPT_PERSIST, persist)
    m = xc.Model(path)
    s = xc.Stage(m, 0, m.n_layer, 256, 8)
    toks, mar, _ = s.decode(p, N_GEN, want_margins=True)
    launches = s.last_decode_launches()[1]
    s.close()
    assert toks.tolist() == want.tolist(), (t, persist)
    assert np.allclose(mar, want_mar, rtol=0.05, atol=2e-3), (t, persist, np.abs(mar - want_mar).max())
    if persist:
        assert launches == 1, "every matrix must be in the tiled layout for the persistent kernel"


def test_typed_model_batch_wider_than_16(xc, typed_model):
    """20 sequences: 20-row GEMVs run as 16-token chunks of the wide kernel."""
    t, path, p, want, _ = typed_model
    m = xc.Model(path)
    rng = np.random.default_rng(7)
    P = rng.integers(0, m.n_vocab, (20, N_PROMPT)).astype(np.int32)
    P[0] = p
    b = xc.Batch(m, 20, 256)
    toks, _, _ = b.decode(P, N_GEN)
    b.close()
    assert toks[0].tolist() == want.tolist(), t
