"""Gated DeltaNet on the GPU: the token-by-token kernel (k_gdn), the chunked prompt kernels
(k_gdn_chunk_prep / k_gdn_chunk / k_gdn_gnorm) and the batch decode kernel (k_gdn_batch) against the
oracle's restatement of the recurrence (oracle/xj_oracle.py:gdn_recurrence, core/xj_cpu.c:194-219) at
the microbenchmark's shape (16 heads, S = 128: prefill of 4096 tokens, decode of 1 and 64 sequences);
the chunked kernels against the token-by-token kernel over more shapes; and prompt forwards that take
the chunked path against the reference's greedy ids."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err
from oracle import xj_oracle as xo

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


# fp32 kernels against the float64 restatement: the chunked form sums in another order and takes exp
# of summed log decays; the token-by-token and batch kernels follow the recurrence step by step
GDN_TOL = 2e-4


def gdn_operands(rng, T, Hk, Hv, S):
    """The microbenchmark's operands: q, k, v and the gate z fp16-representable N(0, 1) (the kernel
    L2-normalises q and k), beta / alpha logits N(0, 1), dt = 0.5 N, A = -exp(0.5 N), norm weights
    1 + 0.1 N (the synthetic models' conventions)."""
    h = lambda *shape: rng.standard_normal(shape).astype(np.float16).astype(np.float32)
    return dict(qkv=h(T, 2 * Hk * S + Hv * S), z=h(T, Hv * S),
                beta=rng.standard_normal((T, Hv)).astype(np.float32),
                alpha=rng.standard_normal((T, Hv)).astype(np.float32),
                dt=(0.5 * rng.standard_normal(Hv)).astype(np.float32),
                A=(-np.exp(0.5 * rng.standard_normal(Hv))).astype(np.float32),
                norm_w=(1 + 0.1 * rng.standard_normal(S)).astype(np.float32))


@pytest.fixture(scope="module")
def prefill_case():
    S, Hk, Hv, T = 128, 16, 16, 4096
    rng = np.random.default_rng(4096)
    op = gdn_operands(rng, T, Hk, Hv, S)
    M0 = (0.05 * rng.standard_normal((Hv, S, S))).astype(np.float32)
    M = M0.astype(np.float64)
    want = xo.gdn_recurrence(op["qkv"], op["z"], op["beta"], op["alpha"], op["dt"].astype(np.float64),
                             op["A"].astype(np.float64), op["norm_w"].astype(np.float64), M, Hk, Hv, S, 1e-6)
    return S, Hk, Hv, op, M0, want, M


@pytest.mark.parametrize("path", [0, 1])
def test_gdn_prefill_4096_matches_oracle(prefill_case, path):
    """16 heads x 128 x 128 state over 4096 tokens from a nonzero state: the token-by-token kernel (path
    0) and the chunked prefill kernels (path 1) against the float64 recurrence."""
    from xjb200 import xjcuda
    S, Hk, Hv, op, M0, want, want_M = prefill_case
    out, M = xjcuda.gdn_run(path, S, Hk, Hv, op["qkv"], op["z"], op["beta"], op["alpha"], op["dt"], op["A"],
                            op["norm_w"], M0)
    assert rel_err(out, want) < GDN_TOL, rel_err(out, want)
    assert rel_err(M, want_M) < GDN_TOL, rel_err(M, want_M)


@pytest.mark.parametrize("B", [1, 64])
def test_gdn_batch_decode_matches_oracle(B):
    """One decode step of B independent sequences (each with its own nonzero state) through the batch
    kernel, against the recurrence run per sequence."""
    from xjb200 import xjcuda
    S, H = 128, 16
    rng = np.random.default_rng(100 + B)
    op = gdn_operands(rng, B, H, H, S)
    M0 = (0.1 * rng.standard_normal((B, H, S, S))).astype(np.float32)
    out, M = xjcuda.gdn_run(2, S, H, H, op["qkv"], op["z"], op["beta"], op["alpha"], op["dt"], op["A"],
                            op["norm_w"], M0)
    for b in range(B):
        Mb = M0[b].astype(np.float64)
        want = xo.gdn_recurrence(op["qkv"][b:b + 1], op["z"][b:b + 1], op["beta"][b:b + 1], op["alpha"][b:b + 1],
                                 op["dt"].astype(np.float64), op["A"].astype(np.float64),
                                 op["norm_w"].astype(np.float64), Mb, H, H, S, 1e-6)
        assert rel_err(out[b:b + 1], want) < GDN_TOL, (b, rel_err(out[b:b + 1], want))
        assert rel_err(M[b], Mb) < GDN_TOL, (b, rel_err(M[b], Mb))
