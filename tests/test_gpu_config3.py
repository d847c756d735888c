"""Parity at the benchmark's own operating point (config 3: 28 layers, E = 2048, Q4_K_M, vocab 151936;
bench.py's 512-token batch-1 prompt). The expected values are the reference's CPU path on the same model
(tests/golden/config3.npz, written by tests/golden/make_config3.py with oracle/_ref):

* 64 greedy ids after the 512-token prompt, through device decode with the persistent kernel and with the
  per-phase kernels, on a stage shaped like the bench's (prompt chunks of 8), and with the prompt in
  chunks of 64 or 512 (tensor-core prompt path);
* activations after every layer and the logits of the first decode step (position 512) through chained
  one-layer stages driven by the vtable with host buffers, within 1e-2 relative (the fp16 KV cache);
* a batch of 64 sequences whose sequence 0 holds the same prompt.

The model is regenerated once per machine into the bench's cache directory (seeded synthetic weights,
about 1.4 GB); its SHA-256 must equal the fixture's, so the expected values belong to it."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_err
from make_config3 import C3_CHUNK, C3_N_CTX, C3_N_GEN, C3_N_PROMPT, file_sha256

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c3():
    return np.load(GOLDEN / "config3.npz")


@pytest.fixture(scope="module")
def config3_path(c3):
    from xjb200 import synth
    p = synth.cached_gguf(synth.CONFIG3, os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models_r0"))
    assert file_sha256(p).tobytes() == c3["c3_sha256"].tobytes(), "regenerated config-3 model differs from the fixture's"
    return p


@pytest.fixture(scope="module")
def model(config3_path):
    from xjb200 import xjcuda
    m = xjcuda.Model(config3_path)
    yield m
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)


@pytest.mark.parametrize("persist", [1, 0])
def test_config3_64_greedy_steps_after_512_prompt(c3, model, persist):
    from xjb200 import xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, persist)
    p = c3["c3_prompt"]
    assert p.size == C3_N_PROMPT
    s = xjcuda.Stage(model, 0, model.n_layer, C3_N_CTX, 8)
    toks, mar, _ = s.decode(p, C3_N_GEN, want_margins=True)
    s.close()
    assert toks.tolist() == c3["c3_tokens"].tolist(), persist
    assert np.allclose(mar, c3["c3_margins"], rtol=0.05, atol=5e-3), (persist, np.abs(mar - c3["c3_margins"]).max())


@pytest.mark.parametrize("chunk", [64, 512])
def test_config3_prompt_in_large_chunks(c3, model, chunk):
    """The same prompt on a stage taking it 64 or 512 tokens at a time: the tcgen05 GEMMs and the chunked
    tensor-core Gated DeltaNet for the prompt, then the persistent kernel, with the reference's 64 ids."""
    from xjb200 import xjcuda
    xjcuda.set_option(xjcuda.OPT_PERSIST, 1)
    s = xjcuda.Stage(model, 0, model.n_layer, C3_N_CTX, chunk)
    toks, mar, _ = s.decode(c3["c3_prompt"], C3_N_GEN, want_margins=True)
    s.close()
    assert toks.tolist() == c3["c3_tokens"].tolist()
    assert np.allclose(mar, c3["c3_margins"], rtol=0.05, atol=5e-3), np.abs(mar - c3["c3_margins"]).max()


def test_config3_layer_trace_at_first_decode_position(c3, model):
    """Per-layer activations and logits of the token at position 512, 1e-2 relative (max |a-b| / max |b|,
    tools/xjpipe-check.c's measure)."""
    from xjb200 import xjcuda
    L = model.n_layer
    stages = [xjcuda.Stage(model, l, l + 1, C3_N_CTX, C3_CHUNK, has_head=(l == L - 1)) for l in range(L)]
    p = np.concatenate([c3["c3_prompt"], c3["c3_tokens"][:1]])
    want_hid, want_lg = c3["c3_trace_hid"], c3["c3_trace_logits"].astype(np.float32)
    chunks = [C3_CHUNK] * (C3_N_PROMPT // C3_CHUNK) + [1]
    pos, x = 0, None
    for c, T in enumerate(chunks):
        x = model.embed_many(p[pos:pos + T])
        for l, s in enumerate(stages):
            x = s.forward(x)
            if c == len(chunks) - 1:
                assert rel_err(x[0], want_hid[l + 1]) < 1e-2, (l, rel_err(x[0], want_hid[l + 1]))
        pos += T
    lg = stages[-1].logits(x)[0]
    assert rel_err(lg, want_lg) < 1e-2, rel_err(lg, want_lg)
    assert int(np.argmax(lg)) == int(c3["c3_tokens"][1])
    for s in stages:
        s.close()


def test_config3_batch_of_64_sequence_0(c3, model):
    from xjb200 import xjcuda
    rng = np.random.default_rng(64)
    P = rng.integers(0, model.n_vocab, (64, C3_N_PROMPT)).astype(np.int32)
    P[0] = c3["c3_prompt"]
    b = xjcuda.Batch(model, 64, C3_N_CTX)
    bt, _, _ = b.decode(P, C3_N_GEN)
    b.close()
    assert bt[0].tolist() == c3["c3_tokens"].tolist()
