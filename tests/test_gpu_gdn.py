"""Gated DeltaNet on the GPU: the chunked prompt kernels (k_gdn_chunk_prep / k_gdn_chunk / k_gdn_gnorm)
against the token-by-token kernel (the recurrence of core/xj_cpu.c:194-219 as written), and prompt
forwards that take the chunked path against the reference's greedy ids."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S,Hk,Hv,T", [(128, 16, 16, 16), (128, 16, 16, 64), (128, 16, 16, 65), (128, 4, 16, 200),
                                       (64, 4, 8, 100), (32, 2, 4, 70), (128, 2, 2, 1000)])
def test_chunked_gdn_matches_token_by_token(S, Hk, Hv, T):
    from xjb200 import xjcuda
    d_out, d_state, ms_c, ms_s = xjcuda.gdn_prefill_check(S, Hk, Hv, T)
    # fp32 both ways; the chunked form sums in another order and takes exp of summed log decays
    assert d_out < 2e-4 and d_state < 2e-4, (d_out, d_state)
    assert ms_c > 0 and ms_s > 0


@pytest.mark.parametrize("which", ["config0", "mid"])
def test_prompt_through_chunked_gdn_gives_reference_ids(golden, config0_path, mid_path, which):
    from make_golden import C0_N_GEN, MID_N_GEN
    from xjb200 import xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)
    m = xjcuda.Model(config0_path if which == "config0" else mid_path)
    p = golden[f"{which}_prompt"]
    n_gen = C0_N_GEN if which == "config0" else MID_N_GEN
    s = xjcuda.Stage(m, 0, m.n_layer, 512, 32)          # prompt forwards of up to 32 tokens: chunked GDN
    toks, _, _ = s.decode(p, n_gen)
    assert toks.tolist() == golden[f"{which}_tokens"].tolist()
    s.close()
