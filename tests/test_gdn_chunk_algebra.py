"""The algebra of the chunked Gated DeltaNet prompt kernels (csrc/kernels.cuh: k_gdn_chunk_prep,
k_gdn_chunk_solve, k_gdn_chunk), restated in float64 numpy on the CPU and checked against the oracle's
token-by-token recurrence (oracle/xj_oracle.py:gdn_recurrence, core/xj_cpu.c:194-219).

Per value head and chunk of tokens with state M0 at its start (G_i: cumulative log decay within the
chunk, b = sigmoid(beta), q and k L2-normalised):
    A[i][l] = b_i e^(G_i - G_l) k_i.k_l (l < i),   T = (I + A)^-1
    W = T diag(b e^G) K,  U0 = T diag(b) V,  D[i][l] = e^(G_i - G_l) q_i.k_l (l <= i)
    Q' = diag(e^G) Q - D W,  O0 = D U0,  Kd[l] = e^(G_C - G_l) k_l
    u = U0 - W M0^T,  o = (O0 + Q' M0^T) / sqrt(S),  M_C = e^(G_C) M0 + u^T Kd
The GPU kernels compute these in fp32 (the products as 3xTF32 tensor-core products); here float64
pins the derivation itself, so the two sides must agree to rounding."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import xj_oracle as xo

C = 64   # tokens per chunk, as GC_C in the kernels


def chunked_gdn(qkv, z, beta, alpha, dt, A, nw, M, Hk, Hv, S, eps):
    """The chunkwise-parallel form over T tokens of one sequence; M [Hv][S][S] updated in place."""
    T = qkv.shape[0]
    kd = Hk * S
    x = qkv.astype(np.float64)
    q = x[:, :kd].reshape(T, Hk, S)
    k = x[:, kd:2 * kd].reshape(T, Hk, S)
    v = x[:, 2 * kd:].reshape(T, Hv, S)
    q = q / np.sqrt((q * q).sum(axis=2, keepdims=True) + eps)
    k = k / np.sqrt((k * k).sum(axis=2, keepdims=True) + eps)
    b_all = 1.0 / (1.0 + np.exp(-beta.astype(np.float64)))
    g_all = np.logaddexp(0.0, alpha.astype(np.float64) + dt) * A
    o_raw = np.zeros((T, Hv, S))
    for hv in range(Hv):
        hk = hv % Hk
        M0 = M[hv].astype(np.float64)
        for t0 in range(0, T, C):
            n = min(C, T - t0)
            K, Q, V = k[t0:t0 + n, hk], q[t0:t0 + n, hk], v[t0:t0 + n, hv]
            b, G = b_all[t0:t0 + n, hv], np.cumsum(g_all[t0:t0 + n, hv])
            dec = np.exp(G[:, None] - G[None, :])
            Am = np.tril(b[:, None] * dec * (K @ K.T), -1)
            Tm = np.linalg.inv(np.eye(n) + Am)
            W = Tm @ ((b * np.exp(G))[:, None] * K)
            U0 = Tm @ (b[:, None] * V)
            D = np.tril(dec * (Q @ K.T))
            Qp = np.exp(G)[:, None] * Q - D @ W
            O0 = D @ U0
            Kd = np.exp(G[-1] - G)[:, None] * K
            u = U0 - W @ M0.T
            o_raw[t0:t0 + n, hv] = (O0 + Qp @ M0.T) / np.sqrt(S)
            M0 = np.exp(G[-1]) * M0 + u.T @ Kd
        M[hv] = M0
    zz = z.astype(np.float64).reshape(T, Hv, S)
    ms = (o_raw * o_raw).mean(axis=2, keepdims=True)
    return (o_raw / np.sqrt(ms + eps) * nw * (zz / (1.0 + np.exp(-zz)))).reshape(T, Hv * S)


@pytest.mark.parametrize("T,Hk,Hv,S", [(150, 2, 4, 32), (64, 1, 2, 16), (33, 2, 2, 16)])
def test_chunked_form_equals_recurrence(T, Hk, Hv, S):
    rng = np.random.default_rng(T + 7 * Hv + S)
    qkv = rng.standard_normal((T, 2 * Hk * S + Hv * S))
    z = rng.standard_normal((T, Hv * S))
    beta, alpha = rng.standard_normal((T, Hv)), rng.standard_normal((T, Hv))
    dt = 0.5 * rng.standard_normal(Hv)
    A = -np.exp(0.5 * rng.standard_normal(Hv))
    nw = 1.0 + 0.1 * rng.standard_normal(S)
    M0 = 0.05 * rng.standard_normal((Hv, S, S))
    M_seq, M_chk = M0.copy(), M0.copy()
    want = xo.gdn_recurrence(qkv, z, beta, alpha, dt, A, nw, M_seq, Hk, Hv, S, 1e-6).astype(np.float64)
    got = chunked_gdn(qkv, z, beta, alpha, dt, A, nw, M_chk, Hk, Hv, S, 1e-6)
    # the oracle returns float32 outputs; the state stays float64 on both sides
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    assert np.abs(M_chk - M_seq).max() <= 1e-10 * np.abs(M_seq).max()
