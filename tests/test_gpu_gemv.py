"""The decode GEMV (y = W x, the reference matmul core/xj_cpu.c:36-54) on the GPU through the C ABI.

Checks, per weight type and shape (the microbenchmark shapes included): fp32-level agreement with a
float64 product of the reference-exact dequantised weights (bound 1e-5 of max|y|: fp32 accumulation,
plus the Q4_K path's codes enter the MMA as 64+q with 64*sum(x) removed afterwards, which costs a few
fp32 ulps of that sum); the tensor-core path equals the generic
path to fp32 rounding; each token's result is bit-identical whatever the number of tokens in the launch
(so decode and speculative verify agree exactly); activations over a wide dynamic range stay exact;
the 64-token kernel of batched decode (17..64 tokens) meets the same bound.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import xj_oracle as xo

pytestmark = pytest.mark.gpu

SHAPES = [(256, 16), (512, 48), (2048, 2048), (2048, 6144), (6144, 2048)]
TYPES = [xo.Q4_K, xo.Q6_K, xo.Q8_0, xo.Q5_K, xo.F16, xo.BF16, xo.F32]


def _w(t, k, n, seed):
    from xjb200 import synth
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    return b"".join(synth.quantize_row(t, x[r]) for r in range(n)) if t != xo.F32 else x.tobytes()


def _ref(t, raw, k, n, x):
    W = xo.dequant(t, raw, k, n).astype(np.float64)
    return x.astype(np.float64) @ W.T


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("k,n", SHAPES)
def test_gemv_matches_float64(t, k, n):
    from xjb200 import xjcuda
    if t in (xo.Q4_K, xo.Q6_K, xo.Q5_K) and k % 256:
        pytest.skip("K-quant rows are whole super-blocks")
    raw = _w(t, k, n, k * 7 + n + t)
    rng = np.random.default_rng(1)
    for T in (1, 3, 4):
        x = rng.standard_normal((T, k)).astype(np.float32)
        want = _ref(t, raw, k, n, x)
        for path in (0, 1):
            y = xjcuda.gemv(t, raw, k, n, x, path)
            err = np.abs(y - want).max() / np.abs(want).max()
            assert err < 1e-5, (t, k, n, T, path, err)


@pytest.mark.parametrize("t", [xo.Q5_K, xo.F16, xo.BF16])
@pytest.mark.parametrize("k,n", [(2048, 2048), (6144, 2048), (2048, 6144)])
def test_gemv_new_tiled_types_wide_and_chunked(t, k, n):
    """Q5_K / F16 / BF16 at 5..16 tokens (the wide kernel) and 20 tokens (16-token chunks)."""
    from xjb200 import xjcuda
    raw = _w(t, k, n, k + 3 * n + t)
    rng = np.random.default_rng(4)
    for T in (5, 16, 20):
        x = rng.standard_normal((T, k)).astype(np.float32)
        want = _ref(t, raw, k, n, x)
        y = xjcuda.gemv(t, raw, k, n, x)
        assert np.abs(y - want).max() / np.abs(want).max() < 1e-5, (t, T)


def test_bf16_outside_scaled_fp16_stays_exact():
    """A BF16 block spanning more than fp16 can carry (1 and 2^-40 side by side) keeps the matrix on
    the row-major kernel; the result still matches the float64 product."""
    from xjb200 import xjcuda
    k, n = 512, 32
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[3, 5] = 1.0
    w[3, 6] = 2.0 ** -40
    raw = (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    x = rng.standard_normal((2, k)).astype(np.float32)
    want = _ref(xo.BF16, raw, k, n, x)
    y = xjcuda.gemv(xo.BF16, raw, k, n, x)
    assert np.abs(y - want).max() / np.abs(want).max() < 1e-5


@pytest.mark.parametrize("t", [xo.Q4_K, xo.Q6_K, xo.Q8_0, xo.Q5_K, xo.F16, xo.BF16])
def test_token_results_independent_of_batch(t):
    from xjb200 import xjcuda
    k, n = 2048, 512
    raw = _w(t, k, n, 3)
    x = np.random.default_rng(2).standard_normal((4, k)).astype(np.float32)
    y4 = xjcuda.gemv(t, raw, k, n, x)
    for i in range(4):
        y1 = xjcuda.gemv(t, raw, k, n, x[i:i + 1])
        assert y1[0].view(np.uint32).tolist() == y4[i].view(np.uint32).tolist()


@pytest.mark.parametrize("t", [xo.Q4_K, xo.Q6_K, xo.Q8_0, xo.Q5_K, xo.F16, xo.BF16])
def test_wide_dynamic_range(t):
    from xjb200 import xjcuda
    k, n = 1024, 64
    raw = _w(t, k, n, 5)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, k)).astype(np.float32)
    x[0] *= 3e4                                    # beyond fp16 range before scaling
    x[1] *= np.exp(rng.uniform(-20, 5, k)).astype(np.float32)   # tiny and large mixed
    want = _ref(t, raw, k, n, x)
    y = xjcuda.gemv(t, raw, k, n, x)
    for r in range(2):
        assert np.abs(y[r] - want[r]).max() / np.abs(want[r]).max() < 1e-5


@pytest.mark.parametrize("t", [xo.Q4_K, xo.Q6_K, xo.Q8_0])
@pytest.mark.parametrize("k,n", [(256, 16), (512, 48), (2048, 2048), (6144, 2048), (2048, 6160)])
@pytest.mark.parametrize("tc", [1, 0])
def test_gemv64_matches_float64(t, k, n, tc):
    """17..64 tokens: the tcgen05 kernel (tc = 1: weights decoded to fp16 hi/lo pairs, f32 accumulator
    in tensor memory) and the mma.sync 64-token kernel (tc = 0); weights once per launch, K split over
    a cluster when the matrix has fewer row blocks than SMs, partial sums added in split order."""
    from xjb200 import xjcuda
    raw = _w(t, k, n, k * 5 + n + t)
    rng = np.random.default_rng(4)
    xjcuda.set_option(xjcuda.OPT_TC, tc)
    try:
        for T in (17, 40, 64):
            x = rng.standard_normal((T, k)).astype(np.float32)
            want = _ref(t, raw, k, n, x)
            y = xjcuda.gemv(t, raw, k, n, x)
            err = np.abs(y - want).max() / np.abs(want).max()
            assert err < 1e-5, (t, k, n, T, tc, err)
    finally:
        xjcuda.set_option(xjcuda.OPT_TC, 1)


@pytest.mark.parametrize("tc", [1, 0])
def test_gemv64_unsplit_many_blocks(tc):
    """More row blocks than SMs: one CTA per block over the whole K (the LM-head case)."""
    from xjb200 import xjcuda
    k, n = 256, 38400
    raw = _w(xo.Q4_K, k, n, 21)
    x = np.random.default_rng(5).standard_normal((33, k)).astype(np.float32)
    want = _ref(xo.Q4_K, raw, k, n, x)
    xjcuda.set_option(xjcuda.OPT_TC, tc)
    try:
        y = xjcuda.gemv(xo.Q4_K, raw, k, n, x)
    finally:
        xjcuda.set_option(xjcuda.OPT_TC, 1)
    assert np.abs(y - want).max() / np.abs(want).max() < 1e-5


@pytest.mark.parametrize("t", [xo.Q4_K, xo.Q6_K, xo.Q8_0])
@pytest.mark.parametrize("tc", [1, 0])
def test_gemv64_token_results_independent_of_batch(t, tc):
    """In both 64-token kernels a token's column depends only on the matrix shape, not on the other
    tokens: the first rows of a 64-token launch equal a 17-token launch bit for bit."""
    from xjb200 import xjcuda
    k, n = 2048, 2048
    raw = _w(t, k, n, 8)
    x = np.random.default_rng(6).standard_normal((64, k)).astype(np.float32)
    xjcuda.set_option(xjcuda.OPT_TC, tc)
    try:
        y64 = xjcuda.gemv(t, raw, k, n, x)
        y17 = xjcuda.gemv(t, raw, k, n, x[:17])
    finally:
        xjcuda.set_option(xjcuda.OPT_TC, 1)
    assert y17.view(np.uint32).tolist() == y64[:17].view(np.uint32).tolist()


@pytest.mark.parametrize("t", [xo.Q6_K, xo.Q4_K, xo.Q8_0])
def test_gemv_lm_head_shape(t):
    """The LM head (151936 x 2048; Q6_K in the Q4_K_M models, the other two types for the microbenchmark)
    at 1, 4 and 16 tokens against the float64 product of the oracle-dequantised weights, every row."""
    from xjb200 import synth, xjcuda
    k, n = 2048, 151936
    rng = np.random.default_rng(151936 + t)
    W = rng.standard_normal(n * k, dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize_row(t, W)
    del W
    D = xo.dequant(t, raw, k, n).astype(np.float64)
    for T in (1, 4, 16):
        x = rng.standard_normal((T, k)).astype(np.float32)
        want = x.astype(np.float64) @ D.T
        y = xjcuda.gemv(t, raw, k, n, x)
        err = np.abs(y - want).max() / np.abs(want).max()
        assert err < 1e-5, (t, T, err)


def test_gemv_microbench_runs():
    from xjb200 import xjcuda
    raw = _w(xo.Q4_K, 2048, 2048, 9)
    ms = xjcuda.gemv_time(xo.Q4_K, raw, 2048, 2048, T=1, copies=4, iters=20)
    assert 0 < ms < 5


def test_gdn_decode_microbench_runs():
    """Gated DeltaNet decode: 16 heads, S = 128, B = 1 and 64 (state 2 MiB per sequence)."""
    from xjb200 import xjcuda
    for B in (1, 64):
        ms = xjcuda.gdn_time(128, 16, B, iters=10)
        assert 0 < ms < 50, (B, ms)
