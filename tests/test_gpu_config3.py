"""Parity at the benchmark's own size (28 layers, E = 2048, Q4_K_M, vocab 151936):
the reference's C implementation (oracle/_ref, core/xj_cpu.c driven by its greedy loop on the host
cores) against device decode through the persistent kernel and the per-phase kernels, and against a
batch that holds the same prompt. The model is generated once per machine into the bench's cache
directory (synthetic seeded weights; about 1.4 GB)."""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PROMPT, N_GEN = 24, 8


@pytest.fixture(scope="module")
def config3_path():
    from xjb200 import synth
    return synth.cached_gguf(synth.CONFIG3, os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models_r0"))


def test_config3_greedy_matches_reference(ref_lib, config3_path):
    from xjb200 import xjcuda, synth
    ref_lib.set_threads(os.cpu_count() or 8)
    rm = ref_lib.Model(config3_path)
    p = np.random.default_rng(2026).integers(0, synth.CONFIG3.n_vocab, N_PROMPT).astype(np.int32)
    want, wmar, _, _ = rm.greedy(p, N_GEN)
    rm.close()
    m = xjcuda.Model(config3_path)
    try:
        for persist in (1, 0):
            xjcuda.set_option(xjcuda.OPT_PERSIST, persist)
            s = xjcuda.Stage(m, 0, m.n_layer, 256, 8)
            toks, mar, _ = s.decode(p, N_GEN, want_margins=True)
            assert toks.tolist() == want.tolist(), persist
            assert np.allclose(mar, wmar, rtol=0.05, atol=2e-3), (persist, np.abs(mar - wmar).max())
            s.close()
        P = np.stack([p, np.roll(p, 5), np.roll(p, 11)])
        b = xjcuda.Batch(m, 3, 256)
        bt, _, _ = b.decode(P, N_GEN)
        assert bt[0].tolist() == want.tolist()
        b.close()
    finally:
        xjcuda.set_option(xjcuda.OPT_PERSIST, 1)
