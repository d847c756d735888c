"""Regenerate tests/golden/config3.npz: reference outputs at the benchmark's operating point.

Run in a checkout that has the reference tree (it is read, never modified) and about 2 GB of disk:

    python tests/golden/make_config3.py [model_dir]

The model is the synthetic ~2B-class hybrid that bench.py times (synth.CONFIG3: 28 layers, E = 2048,
Q4_K_M, vocab 151936), written by the repository's seeded writer; the prompt is bench.py's batch-1
prompt of rank 0 (512 seeded token ids). The reference's own CPU path (oracle/_ref/libxjref.so, its
core/*.c built unchanged) produces:

  c3_sha256          SHA-256 of the model file, so a test can tell that the model it regenerated is
                     the one these outputs belong to
  c3_prompt          the 512 prompt ids
  c3_tokens          64 greedy ids after the prompt (max_batch 64, n_ctx 640)
  c3_margins         the top-2 logit gap of each of those steps
  c3_trace_hid       activations after every layer ([L+1][E], row 0 = embedding) of the first decode
                     step: the prompt in chunks of 64 through one-layer stages, then c3_tokens[0] at
                     position 512 (tools/xjpipe-check.c's chained-stage pattern)
  c3_trace_logits    that step's logits, stored as float16 (their rounding, <= 2^-11 relative, is far
                     below the 1e-2 gate they are checked at)
The GPU box has no reference tree, so the tests read this file.
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import pathlib
import sys
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle import ref  # noqa: E402

# bench.py's batch-1 workload (rank 0) and the parity depth asked of it
C3_PROMPT_SEED, C3_N_PROMPT, C3_N_GEN, C3_CHUNK, C3_N_CTX = 1234, 512, 64, 64, 640


def load_pkg():
    spec = importlib.util.spec_from_file_location("xjb200", ROOT / "meta-work_b200" / "__init__.py",
                                                  submodule_search_locations=[str(ROOT / "meta-work_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xjb200"] = mod
    spec.loader.exec_module(mod)
    return mod


def c3_prompt(vocab: int) -> np.ndarray:
    return np.random.default_rng(C3_PROMPT_SEED).integers(0, vocab, C3_N_PROMPT).astype(np.int32)


def file_sha256(path) -> np.ndarray:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 24), b""):
            h.update(blk)
    return np.frombuffer(h.digest(), np.uint8)


def main():
    if not ref.REF_TREE.exists():
        sys.exit("reference tree not found; the config-3 fixture can only be regenerated where it exists")
    ref.build()
    load_pkg()
    from xjb200 import synth
    mdir = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models_r0")
    path = synth.cached_gguf(synth.CONFIG3, mdir)
    ref.set_threads(os.cpu_count() or 8)
    g = {"c3_sha256": file_sha256(path)}
    m = ref.Model(path)
    p = c3_prompt(m.n_vocab)
    t0 = time.time()
    tok, mar, _, _ = m.greedy(p, C3_N_GEN, max_batch=C3_CHUNK, n_ctx=C3_N_CTX)
    print(f"greedy: {time.time() - t0:.0f} s", flush=True)
    chunks = [C3_CHUNK] * (C3_N_PROMPT // C3_CHUNK) + [1]
    t0 = time.time()
    hid, lg = m.layer_trace(np.concatenate([p, tok[:1]]), chunks, max_batch=C3_CHUNK, n_ctx=C3_N_CTX)
    print(f"layer trace: {time.time() - t0:.0f} s", flush=True)
    assert int(np.argmax(lg[0])) == int(tok[1])
    g.update(c3_prompt=p, c3_tokens=tok, c3_margins=mar, c3_trace_hid=hid[:, 0, :].copy(),
             c3_trace_logits=lg[0].astype(np.float16))
    m.close()
    np.savez_compressed(HERE / "config3.npz", **g)
    print("wrote", HERE / "config3.npz")


if __name__ == "__main__":
    main()
