"""Regenerate the committed golden fixtures from the reference implementation.

Run in a checkout that has the reference tree (it is read, never modified):

    python tests/golden/make_golden.py

Writes, next to this script:
  tiny_mtp.gguf   the reference's own synthetic test model, produced by running the reference's
                  src/xiaoju-pipe/tests/make_tiny_model.py --mtp unchanged (8 layers, E=64, mixed
                  F32 / Q8_0 weights, vocab 288, one MTP layer, seed 20261107).
  golden.npz      outputs of the reference CPU path (oracle/_ref/libxjref.so, built from the
                  reference's own core/*.c by oracle/Makefile) on that model and on the synthetic
                  config-0 (Q8_0) and mid (Q4_K_M, config-3 head shapes) models, plus row
                  dequantisation known answers for every supported type.
The GPU box has no reference tree, so the tests read these files instead of re-running the reference.
"""
from __future__ import annotations

import hashlib
import importlib.util
import pathlib
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle import ref  # noqa: E402

REF_TREE = ref.REF_TREE


def load_pkg():
    spec = importlib.util.spec_from_file_location("xjb200", ROOT / "meta-work_b200" / "__init__.py",
                                                  submodule_search_locations=[str(ROOT / "meta-work_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xjb200"] = mod
    spec.loader.exec_module(mod)
    return mod


# Seeds and shapes of every golden case (tests import these so they never drift apart).
TINY_PROMPT_SEED, TINY_N_PROMPT, TINY_N_GEN = 7, 24, 48
C0_PROMPT_SEED, C0_N_PROMPT, C0_N_GEN = 1, 32, 64
MID_PROMPT_SEED, MID_N_PROMPT, MID_N_GEN = 3, 40, 64
TRACE_CHUNKS = (12, 1, 1, 1)      # tools/xjpipe-check.c:61 (prefill 12, then 3 single tokens)
DQ_ROWS, DQ_K = 4, 512


def prompt(seed: int, n: int, vocab: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


def dequant_cases(synth):
    """Raw rows per type: 2 rows quantised from N(0, 0.02) data + 2 rows of random bytes (block scales
    forced finite), so every bit pattern path of the decoders is exercised."""
    rng = np.random.default_rng(99)
    out = {}
    for t, (bn, bb) in {synth.F16: (1, 2), synth.BF16: (1, 2), synth.Q8_0: (32, 34), synth.Q4_K: (256, 144),
                        synth.Q5_K: (256, 176), synth.Q6_K: (256, 210)}.items():
        rows = []
        for r in range(2):
            rows.append(np.frombuffer(synth.quantize_row(t, rng.standard_normal(DQ_K).astype(np.float32) * 0.02), np.uint8))
        for r in range(2):
            raw = rng.integers(0, 256, DQ_K // bn * bb).astype(np.uint8)
            if t in (synth.F16,):
                raw = raw.view(np.uint16)
                raw &= 0xBBFF                                     # keep exponents small and finite
                raw = raw.view(np.uint8)
            elif t == synth.BF16:
                raw = raw.view(np.uint16)
                raw = ((raw & 0x807F) | 0x3C00).astype(np.uint16).view(np.uint8)
            else:
                blk = raw.reshape(-1, bb)
                fpos = {synth.Q8_0: [0], synth.Q4_K: [0, 2], synth.Q5_K: [0, 2], synth.Q6_K: [208]}[t]
                for p in fpos:                                    # fp16 scale fields: |x| < 2, finite
                    h = blk[:, p:p + 2].copy().view(np.uint16)
                    h &= 0xBBFF
                    blk[:, p:p + 2] = h.view(np.uint8).reshape(-1, 2)
                raw = blk.reshape(-1)
            rows.append(raw.astype(np.uint8))
        raw = np.concatenate(rows)
        dq = np.stack([ref.dequant_row(t, raw[i * len(raw) // DQ_ROWS:(i + 1) * len(raw) // DQ_ROWS], DQ_K)
                       for i in range(DQ_ROWS)])
        out[t] = (raw, dq)
    return out


def main():
    if not REF_TREE.exists():
        sys.exit("reference tree not found; golden fixtures can only be regenerated where it exists")
    ref.build()
    pkg = load_pkg()
    from xjb200 import synth
    tiny = HERE / "tiny_mtp.gguf"
    subprocess.run([sys.executable, str(REF_TREE / "tests" / "make_tiny_model.py"), str(tiny), "--mtp"], check=True,
                   cwd=str(REF_TREE))
    g = {}
    # ---- reference tiny model ----
    m = ref.Model(tiny)
    p = prompt(TINY_PROMPT_SEED, TINY_N_PROMPT, m.n_vocab)
    tok, mar, first, _ = m.greedy(p, TINY_N_GEN, max_batch=8, n_ctx=512)
    hid, lg = m.layer_trace(p[:sum(TRACE_CHUNKS)], TRACE_CHUNKS, max_batch=16, n_ctx=128)
    g.update(tiny_prompt=p, tiny_tokens=tok, tiny_margins=mar, tiny_first_logits=first, tiny_trace_hid=hid,
             tiny_trace_logits=lg, tiny_fingerprint=np.uint64(m.fingerprint))
    for k in (0, 1, 3, 4):
        st, stats = m.spec(p, TINY_N_GEN, k, max_batch=8, n_ctx=512)
        g[f"tiny_spec_k{k}"] = st
        g[f"tiny_spec_k{k}_stats"] = stats
    st, _ = m.spec(p, TINY_N_GEN, 0, max_batch=8, n_ctx=512, s1=3)
    g["tiny_split3"] = st
    m.close()
    # the synthetic models are not fixtures: they live in a temporary directory removed at the end
    with tempfile.TemporaryDirectory(prefix="xj_golden_") as tmpdir:
        synthetic_cases(g, synth, pathlib.Path(tmpdir))
    # ---- dequant known answers ----
    for t, (raw, dq) in dequant_cases(synth).items():
        g[f"dq_{t}_raw"] = raw
        g[f"dq_{t}_f32"] = dq
    np.savez_compressed(HERE / "golden.npz", **g)
    print("wrote", HERE / "golden.npz", "and", tiny)


def synthetic_cases(g, synth, tmp: pathlib.Path):
    """Reference outputs on the synthetic config-0 (Q8_0) and mid (Q4_K_M) models written into tmp."""
    # ---- synthetic config 0 ----
    c0 = tmp / "golden_config0.gguf"
    synth.write_gguf(c0, synth.CONFIG0)
    g["config0_sha256"] = np.frombuffer(hashlib.sha256(c0.read_bytes()).digest(), np.uint8)
    m0 = ref.Model(c0)
    p0 = prompt(C0_PROMPT_SEED, C0_N_PROMPT, m0.n_vocab)
    tok0, mar0, first0, _ = m0.greedy(p0, C0_N_GEN, max_batch=8, n_ctx=512)
    hid0, lg0 = m0.layer_trace(p0[:sum(TRACE_CHUNKS)], TRACE_CHUNKS, max_batch=16, n_ctx=128)
    g.update(config0_prompt=p0, config0_tokens=tok0, config0_margins=mar0, config0_first_logits=first0,
             config0_trace_hid=hid0, config0_trace_logits=lg0, config0_fingerprint=np.uint64(m0.fingerprint))
    # ---- synthetic mid model (Q4_K / Q6_K, 128-wide heads) ----
    cm = tmp / "golden_mid.gguf"
    synth.write_gguf(cm, synth.MID)
    g["mid_sha256"] = np.frombuffer(hashlib.sha256(cm.read_bytes()).digest(), np.uint8)
    mm = ref.Model(cm)
    pm = prompt(MID_PROMPT_SEED, MID_N_PROMPT, mm.n_vocab)
    tokm, marm, firstm, _ = mm.greedy(pm, MID_N_GEN, max_batch=8, n_ctx=512)
    g.update(mid_prompt=pm, mid_tokens=tokm, mid_margins=marm, mid_first_logits=firstm,
             mid_fingerprint=np.uint64(mm.fingerprint))
    m0.close()
    mm.close()


if __name__ == "__main__":
    main()
