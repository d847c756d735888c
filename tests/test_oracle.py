"""Pins the numpy oracle (oracle/xj_oracle.py) to the reference: known answers from the reference unit
tests, bit-exact dequantisation against golden vectors written by the reference, and whole-model
greedy decoding / activations against the reference's own outputs. CPU only."""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from conftest import rel_err
from make_golden import (C0_N_GEN, C0_N_PROMPT, C0_PROMPT_SEED, DQ_K, DQ_ROWS, TINY_N_GEN, TRACE_CHUNKS,
                         prompt)
from oracle import xj_oracle as xo

TYPES = (xo.F16, xo.BF16, xo.Q8_0, xo.Q4_K, xo.Q5_K, xo.Q6_K)


def f16_bits(v: float) -> int:
    return int(np.array([v], np.float16).view(np.uint16)[0])


def test_f16_roundtrip_known_answers():
    # src/xiaoju-pipe/tests/unit.c:17-25
    for v in (0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.9604645e-08, 0.33325195, -1e-3):
        back = float(xo.f16(np.array([f16_bits(v)], np.uint16))[0])
        assert abs(back - v) <= abs(v) * 1e-3 + 1e-7
    assert np.isinf(xo.f16(np.array([f16_bits(1e6)], np.uint16))[0])


def test_q8_0_known_answer():
    # unit.c:27-34: d = 0.5, q[i] = i - 16
    b = struct.pack("<H", f16_bits(0.5)) + bytes((i - 16) & 0xFF for i in range(32))
    y = xo.dequant(xo.Q8_0, b, 32)[0]
    assert np.array_equal(y, 0.5 * (np.arange(32) - 16).astype(np.float32))


def _q4k_kat_block() -> bytes:
    # unit.c:36-42: d = 0.25, dmin = 1; sub-blocks 0..3 scale j+1 / min j, sub-blocks 4..7 scale 2 / min 1
    b = bytearray(144)
    b[0:2] = struct.pack("<H", f16_bits(0.25))
    b[2:4] = struct.pack("<H", f16_bits(1.0))
    for j in range(4):
        b[4 + j] = j + 1
        b[8 + j] = j
    for j in range(4, 8):
        b[12 + j - 4] = 2 | (1 << 4)
    for i in range(128):
        b[16 + i] = (i % 16) | ((15 - i % 16) << 4)
    return bytes(b)


def test_q4_k_known_answer():
    # unit.c:43-51, including the high-bit scale path of sub-blocks 4..7
    b = _q4k_kat_block()
    y = xo.dequant(xo.Q4_K, b, 256)[0]
    for e in range(256):
        j, l, g = e // 32, e % 32, (e // 32) // 2
        q = (b[16 + 32 * g + l] >> 4) if (j & 1) else (b[16 + 32 * g + l] & 15)
        sc, mn = (j + 1, j) if j < 4 else (2, 1)
        assert abs(y[e] - (0.25 * sc * q - 1.0 * mn)) < 1e-6


def test_known_answers_match_live_reference(ref_lib):
    b = _q4k_kat_block()
    assert np.array_equal(ref_lib.dequant_row(xo.Q4_K, b, 256), xo.dequant(xo.Q4_K, b, 256)[0])
    for v in (0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.9604645e-08, 0.33325195, -1e-3, 1e6):
        assert ref_lib.f32_to_f16(v) == f16_bits(v)


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_vs_golden(golden, t):
    raw, want = golden[f"dq_{t}_raw"], golden[f"dq_{t}_f32"]
    got = xo.dequant(t, raw.tobytes(), DQ_K, DQ_ROWS)
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_vs_live_reference(ref_lib, t):
    from xjb200 import synth
    rng = np.random.default_rng(t)
    x = (rng.standard_normal(4096) * rng.choice([0.02, 1.0, 50.0])).astype(np.float32)
    raw = synth.quantize_row(t, x)
    assert ref_lib.dequant_row(t, raw, 4096).view(np.uint32).tolist() == \
        xo.dequant(t, raw, 4096)[0].view(np.uint32).tolist()


def test_quantizers_round_trip():
    from xjb200 import synth
    x = (np.random.default_rng(3).standard_normal(2048) * 0.02).astype(np.float32)
    tol = {xo.Q8_0: 0.01, xo.Q4_K: 0.12, xo.Q5_K: 0.06, xo.Q6_K: 0.03, xo.F16: 1e-3, xo.BF16: 8e-3}
    for t, r in tol.items():
        y = xo.dequant(t, synth.quantize_row(t, x), 2048)[0]
        assert np.abs(y - x).max() <= r * np.abs(x).max(), t


def test_synth_model_is_deterministic(golden, config0_path):
    assert hashlib.sha256(config0_path.read_bytes()).digest() == golden["config0_sha256"].tobytes()


def test_oracle_greedy_matches_reference_tiny(golden, tiny_path):
    m = xo.Model(tiny_path)
    toks = xo.greedy(m, golden["tiny_prompt"], TINY_N_GEN, max_batch=8, n_ctx=512)
    assert toks.tolist() == golden["tiny_tokens"].tolist()


def test_oracle_greedy_matches_reference_config0(golden, config0_path):
    m = xo.Model(config0_path)
    p = prompt(C0_PROMPT_SEED, C0_N_PROMPT, m.hp.n_vocab)
    assert p.tolist() == golden["config0_prompt"].tolist()
    toks = xo.greedy(m, p, C0_N_GEN, max_batch=8, n_ctx=512)
    assert toks.tolist() == golden["config0_tokens"].tolist()


@pytest.mark.parametrize("which", ["tiny", "config0"])
def test_oracle_layer_trace_matches_reference(golden, tiny_path, config0_path, which):
    m = xo.Model(tiny_path if which == "tiny" else config0_path)
    p = golden[f"{which}_prompt"]
    want_hid, want_lg = golden[f"{which}_trace_hid"], golden[f"{which}_trace_logits"]
    stages = [xo.Stage(m, l, l + 1, 128, 16, has_head=(l == m.hp.n_layer - 1)) for l in range(m.hp.n_layer)]
    pos = 0
    for c, T in enumerate(TRACE_CHUNKS):
        x = np.stack([m.embed(int(t)) for t in p[pos:pos + T]])
        for l, s in enumerate(stages):
            x = s.forward(x)
            if c == len(TRACE_CHUNKS) - 1:
                assert rel_err(x, want_hid[l + 1]) < 1e-4, (which, l)
        pos += T
    assert rel_err(stages[-1].logits(x), want_lg) < 1e-4


def test_oracle_rollback_equivalence(tiny_path):
    # tools/xjpipe-check.c:78-109: forward 6, forward 4 with keep, roll back to 8, forward 2 new
    # == a fresh run over the same 10 tokens.
    m = xo.Model(tiny_path)
    toks = prompt(11, 16, m.hp.n_vocab)
    E = lambda ids: np.stack([m.embed(int(t)) for t in ids])
    s = xo.Stage(m, 0, m.hp.n_layer, 64, 16)
    s.forward(E(toks[:6]))
    s.keep = 4
    s.forward(E(toks[6:10]))
    assert (s.ck_start, s.ck_T) == (6, 4)
    s.rollback(8)
    out = s.forward(E(toks[12:14]))
    f = xo.Stage(m, 0, m.hp.n_layer, 64, 16)
    want = f.forward(E(np.concatenate([toks[:8], toks[12:14]])))[-2:]
    assert rel_err(out, want) < 1e-5
    with pytest.raises(ValueError):
        s.rollback(3)


def test_gdn_recurrence_matches_float32_token_step():
    """The vectorised float64 recurrence (the GPU GDN tests' reference) against the float32 per-token
    step that the oracle's attn_linear uses (itself pinned to the reference by the greedy and layer-trace
    tests above), over 48 tokens of 2 key / 4 value heads."""
    rng = np.random.default_rng(5)
    T, Hk, Hv, S, eps = 48, 2, 4, 16, 1e-6
    qkv = rng.standard_normal((T, 2 * Hk * S + Hv * S)).astype(np.float32)
    z = rng.standard_normal((T, Hv * S)).astype(np.float32)
    beta = rng.standard_normal((T, Hv)).astype(np.float32)
    alpha = rng.standard_normal((T, Hv)).astype(np.float32)
    dt = (0.5 * rng.standard_normal(Hv)).astype(np.float32)
    A = (-np.exp(0.5 * rng.standard_normal(Hv))).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(S)).astype(np.float32)
    M0 = (0.1 * rng.standard_normal((Hv, S, S))).astype(np.float32)
    M64 = M0.astype(np.float64)
    want = xo.gdn_recurrence(qkv, z, beta, alpha, dt.astype(np.float64), A.astype(np.float64),
                             nw.astype(np.float64), M64, Hk, Hv, S, eps)
    M32 = M0.copy()
    qs = np.float32(1.0 / np.sqrt(np.float32(S)))
    got = np.stack([xo.gdn_token(qkv[t, :Hk * S].reshape(Hk, S), qkv[t, Hk * S:2 * Hk * S].reshape(Hk, S),
                                 qkv[t, 2 * Hk * S:].reshape(Hv, S), beta[t], alpha[t], z[t], dt, A, nw, M32,
                                 Hk, Hv, S, eps, qs) for t in range(T)])
    assert rel_err(got, want) < 1e-5
    assert rel_err(M32, M64) < 1e-5


def test_config3_fixture_is_consistent():
    """tests/golden/config3.npz (the reference at the benchmark's operating point) holds bench.py's
    prompt, 64 ids, and a last-step trace whose logits pick the second id."""
    from make_config3 import C3_N_GEN, C3_N_PROMPT, c3_prompt
    from conftest import GOLDEN
    c3 = np.load(GOLDEN / "config3.npz")
    assert c3["c3_prompt"].tolist() == c3_prompt(151936).tolist() and c3["c3_prompt"].size == C3_N_PROMPT
    assert c3["c3_tokens"].size == C3_N_GEN and c3["c3_margins"].size == C3_N_GEN
    assert c3["c3_trace_hid"].shape == (29, 2048)
    assert int(np.argmax(c3["c3_trace_logits"].astype(np.float32))) == int(c3["c3_tokens"][1])
