"""The tcgen05 building blocks of the batched kernels: shared-memory matrix descriptors, the fp16 MMA
with an f32 accumulator in tensor memory and the tensor-memory read-back, against numpy."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", [64, 256, 2048])
def test_tc_selftest_matches_numpy(k):
    from xjb200 import xjcuda as xc
    rng = np.random.default_rng(k)
    a = rng.standard_normal((128, k)).astype(np.float16)
    b = rng.standard_normal((64, k)).astype(np.float16)
    d = xc.tc_selftest(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    # fp16 products are exact in f32; only the f32 accumulation rounds
    np.testing.assert_allclose(d, ref, rtol=0, atol=1e-5 * np.sqrt(k) * 8)
