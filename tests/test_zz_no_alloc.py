"""The allocation-free entry point, xj_cuda_norm_gemv_noalloc, against the regular one.

Some callers cannot allocate device memory where they need this product (a fixed memory pool owned by
another component, or a thread on which cudaMalloc is not allowed). xj_cuda_norm_gemv_noalloc takes
device pointers for every input and output and keeps its one intermediate, the RMS-normalised rows, in
a fixed device array inside the library. Its result must match the regular xj_cuda_gemv (which copies
host buffers into memory it allocates) applied to the same rows normalised on the host, for two calls
in a row, since the fixed array keeps the previous call's contents.

This file sorts last so that, in a run that stops at the first failure, every other test has run; it
passes alone in a fresh process as well. Device buffers come from torch, which shares the device's
primary context with the library.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_K, Q8_0 = 12, 8


def host_rmsnorm(x, w, eps):
    ss = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    sc = (np.float32(1) / np.sqrt((ss / x.shape[1]).astype(np.float32) + np.float32(eps))).astype(np.float32)
    return ((x * sc) * w).astype(np.float32)


@pytest.mark.parametrize("t,k,n", [(Q4_K, 2048, 512), (Q8_0, 1408, 96)])
def test_noalloc_matches_regular_entry_point_twice(t, k, n):
    import torch
    from xjb200 import synth, xjcuda
    lib = xjcuda.lib()
    rng = np.random.default_rng(7)
    raw = b"".join(synth.quantize_row(t, (rng.standard_normal(k) * 0.02).astype(np.float32)) for _ in range(n))
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    eps = 1e-6
    w_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()
    nw_dev = torch.from_numpy(nw).cuda()
    err = ctypes.create_string_buffer(512)
    for call, T in enumerate((3, 1)):
        x = (rng.standard_normal((T, k)) * (1 + call)).astype(np.float32)
        x_dev = torch.from_numpy(x).cuda()
        y_dev = torch.full((T, n), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        rc = lib.xj_cuda_norm_gemv_noalloc(t, w_dev.data_ptr(), k, n, x_dev.data_ptr(), nw_dev.data_ptr(), eps, T,
                                           y_dev.data_ptr(), err, 512)
        assert rc == 0, err.value.decode()
        got = y_dev.cpu().numpy()
        want = xjcuda.gemv(t, raw, k, n, host_rmsnorm(x, nw, eps), path=1)
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() / np.abs(want).max() < 1e-5, (call, T)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    from xjb200 import xjcuda
    lib = xjcuda.lib()
    k, n, T = 8192, 16, 16                     # T*k = 131072 floats > the 65536-float scratch
    w_dev = torch.zeros(n * k // 32 * 34, dtype=torch.uint8, device="cuda")
    x_dev = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    nw_dev = torch.ones(k, dtype=torch.float32, device="cuda")
    y_dev = torch.zeros((T, n), dtype=torch.float32, device="cuda")
    err = ctypes.create_string_buffer(512)
    rc = lib.xj_cuda_norm_gemv_noalloc(Q8_0, w_dev.data_ptr(), k, n, x_dev.data_ptr(), nw_dev.data_ptr(), 1e-6, T,
                                       y_dev.data_ptr(), err, 512)
    assert rc == -1 and b"scratch" in err.value
