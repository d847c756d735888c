"""numpy restatement of the xiaoju-pipe CPU path (the oracle for the CUDA stage).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may use it,
as the checker, never as the measured or shipped path.

Every function restates one piece of the reference and cites it (paths relative to
src/xiaoju-pipe/):

- f16 / bf16 decoding                 core/xj_quant.h:9-45
- 6-bit K-quant scale/min unpacking   core/xj_quant.h:49-52
- row dequantisation (all types)      core/xj_quant.h:55-122
- GGUF v2/v3 header parsing           core/gguf.c:106-186
- hparams + layer table               core/xj_model.c:62-202
- matmul / rmsnorm / rope             core/xj_cpu.c:36-77
- gated full attention                core/xj_cpu.c:83-151
- Gated DeltaNet                      core/xj_cpu.c:155-223
- layer loop, head, rollback, reset   core/xj_cpu.c:228-330
- embedding lookup                    core/xj_cpu.c:369-373

Pinning: tests/test_oracle.py checks this module against the reference library built from the
reference sources (oracle/_ref, when present) and against the committed golden vectors in
tests/golden/ (produced by that library), plus the reference unit-test known answers
(tests/unit.c:17-52).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 30

# elements per block, bytes per block (core/gguf.c:12-32)
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
         Q8_0: (32, 34), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
SUPPORTED = (F32, F16, BF16, Q8_0, Q4_K, Q5_K, Q6_K)   # core/xj_model.c:16-17


def row_bytes(t: int, n: int) -> int:
    bn, bb = BLOCK[t]
    return n // bn * bb


# ---------------------------------------------------------------- dequantisation (xj_quant.h)
def f16(u: np.ndarray) -> np.ndarray:
    """IEEE half -> float32, exact (xj_quant.h:9-23)."""
    return np.asarray(u, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16(u: np.ndarray) -> np.ndarray:
    """bfloat16 -> float32 (xj_quant.h:45)."""
    return (np.asarray(u, dtype=np.uint32) << 16).view(np.float32)


def scale_min_k4(q: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Unpack the 12-byte scale field of [nb] K-quant blocks into sc[nb][8], m[nb][8] (xj_quant.h:49-52)."""
    q = q.astype(np.uint8)
    sc = np.empty(q.shape[:-1] + (8,), np.uint8)
    mn = np.empty_like(sc)
    sc[..., :4] = q[..., 0:4] & 63
    mn[..., :4] = q[..., 4:8] & 63
    sc[..., 4:] = (q[..., 8:12] & 0xF) | ((q[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (q[..., 8:12] >> 4) | ((q[..., 4:8] >> 6) << 4)
    return sc, mn


def dequant(t: int, raw, n: int, rows: int = 1) -> np.ndarray:
    """Decode `rows` rows of `n` elements of type `t` to float32 [rows][n] (xj_quant.h:55-122).

    Uses the reference's own float32 operation order per element (d*sc then *q, minus dmin*m), so the
    result is bit-identical to xj_dequant_row.
    """
    b = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).ravel()
    if t == F32:
        return b[:rows * n * 4].view(np.float32).reshape(rows, n).copy()
    if t == F16:
        return f16(b[:rows * n * 2].view(np.uint16)).reshape(rows, n)
    if t == BF16:
        return bf16(b[:rows * n * 2].view(np.uint16)).reshape(rows, n)
    nb = rows * n // BLOCK[t][0]
    blk = b[:nb * BLOCK[t][1]].reshape(nb, BLOCK[t][1])
    if t == Q8_0:
        d = f16(blk[:, 0:2].copy().view(np.uint16))            # [nb,1]
        q = blk[:, 2:].view(np.int8).astype(np.float32)         # [nb,32]
        return (d * q).astype(np.float32).reshape(rows, n)
    if t in (Q4_K, Q5_K):
        d = f16(blk[:, 0:2].copy().view(np.uint16))             # [nb,1]
        dmin = f16(blk[:, 2:4].copy().view(np.uint16))
        sc, mn = scale_min_k4(blk[:, 4:16])
        d1 = (d * sc.astype(np.float32)).astype(np.float32)     # [nb,8]  d*sc  (float)
        m1 = (dmin * mn.astype(np.float32)).astype(np.float32)  # [nb,8]  dmin*m
        if t == Q4_K:
            qs = blk[:, 16:144].reshape(nb, 4, 32)
            lo, hi = qs & 0xF, qs >> 4
            q = np.stack([lo, hi], axis=2).reshape(nb, 8, 32)   # sub-block 2g = low nibbles, 2g+1 = high
        else:
            qh = blk[:, 16:48]                                   # [nb,32]
            ql = blk[:, 48:176].reshape(nb, 4, 32)
            q = np.empty((nb, 8, 32), np.uint8)
            for g in range(4):
                q[:, 2 * g] = (ql[:, g] & 0xF) + np.where(qh & (1 << (2 * g)), 16, 0)
                q[:, 2 * g + 1] = (ql[:, g] >> 4) + np.where(qh & (2 << (2 * g)), 16, 0)
        y = d1[:, :, None] * q.astype(np.float32) - m1[:, :, None]
        return y.astype(np.float32).reshape(rows, n)
    if t == Q6_K:
        ql = blk[:, 0:128].reshape(nb, 2, 64)
        qh = blk[:, 128:192].reshape(nb, 2, 32)
        sc = blk[:, 192:208].view(np.int8).reshape(nb, 2, 8).astype(np.float32)
        d = f16(blk[:, 208:210].copy().view(np.uint16)).reshape(nb, 1, 1)
        y = np.empty((nb, 2, 128), np.float32)
        l = np.arange(32)
        isx = l // 16
        parts = [
            ((ql[:, :, 0:32] & 0xF) | ((qh >> 0) & 3) << 4, 0),
            ((ql[:, :, 32:64] & 0xF) | ((qh >> 2) & 3) << 4, 2),
            ((ql[:, :, 0:32] >> 4) | ((qh >> 4) & 3) << 4, 4),
            ((ql[:, :, 32:64] >> 4) | ((qh >> 6) & 3) << 4, 6),
        ]
        for w, (qv, so) in enumerate(parts):
            qi = qv.astype(np.int32) - 32
            s = sc[:, :, isx + so]                               # [nb,2,32]
            y[:, :, 32 * w:32 * w + 32] = ((d * s).astype(np.float32) * qi.astype(np.float32))
        return y.astype(np.float32).reshape(rows, n)
    return np.zeros((rows, n), np.float32)                     # unsupported -> zeros (xj_quant.h:120)


# ---------------------------------------------------------------- GGUF (gguf.c:106-186)
_VSIZE = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
_VFMT = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}


@dataclass
class Tensor:
    name: str
    ne: list
    type: int
    offset: int
    nbytes: int


@dataclass
class Gguf:
    kv: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    data_off: int = 0
    buf: object = None

    def data(self, t: Tensor) -> np.ndarray:
        return np.frombuffer(self.buf, dtype=np.uint8, count=t.nbytes, offset=self.data_off + t.offset)


def read_gguf(path: str | os.PathLike) -> Gguf:
    f = open(path, "rb")
    buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    p = 0

    def rd(fmt):
        nonlocal p
        v = struct.unpack_from("<" + fmt, buf, p)
        p += struct.calcsize("<" + fmt)
        return v[0]

    def rs():
        n = rd("Q")
        nonlocal p
        s = bytes(buf[p:p + n]).decode("utf-8", "replace")
        p += n
        return s

    def val(t):
        if t == 8:
            return rs()
        if t == 9:
            at, n = rd("I"), rd("Q")
            return [val(at) for _ in range(n)]
        return rd(_VFMT[t])

    magic, version = rd("I"), rd("I")
    if magic != 0x46554747 or version not in (2, 3):
        raise ValueError("not a GGUF v2/v3 file")
    n_t, n_kv = rd("Q"), rd("Q")
    g = Gguf(buf=buf)
    align = 32
    for _ in range(n_kv):
        k = rs()
        t = rd("I")
        g.kv[k] = val(t)
        if k == "general.alignment":
            align = int(g.kv[k])
    for _ in range(n_t):
        name = rs()
        nd = rd("I")
        ne = [rd("Q") for _ in range(nd)] + [1] * (4 - nd)
        t = rd("I")
        off = rd("Q")
        nb = row_bytes(t, ne[0]) * ne[1] * ne[2] * ne[3] if t in BLOCK else 0
        g.tensors[name] = Tensor(name, ne, t, off, nb)
    g.data_off = (p + align - 1) // align * align
    return g


# ---------------------------------------------------------------- model (xj_model.c)
@dataclass
class HParams:
    n_layer: int
    n_embd: int
    n_ff: int
    n_vocab: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_rot: int
    rope_base: float
    eps: float
    conv_k: int
    d_inner: int
    s_k: int
    h_k: int
    h_v: int

    @property
    def s_v(self):
        return self.d_inner // self.h_v

    @property
    def key_dim(self):
        return self.s_k * self.h_k

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.d_inner


class Weight:
    """A weight tensor; .f32 dequantises the whole matrix once ([ne1][ne0])."""

    def __init__(self, g: Gguf, t: Tensor):
        self.g, self.t = g, t
        self.type, self.ne0 = t.type, t.ne[0]
        self.ne1 = t.ne[1] * t.ne[2] * t.ne[3]
        self._f = None

    @property
    def raw(self) -> np.ndarray:
        return self.g.data(self.t)

    @property
    def f32(self) -> np.ndarray:
        if self._f is None:
            self._f = dequant(self.type, self.raw, self.ne0, self.ne1)
        return self._f

    def row(self, r: int) -> np.ndarray:
        rb = row_bytes(self.type, self.ne0)
        return dequant(self.type, self.raw[r * rb:(r + 1) * rb], self.ne0)[0]


class Model:
    """Hparams + weights of a qwen35 GGUF (core/xj_model.c:129-202)."""

    def __init__(self, path):
        g = self.g = read_gguf(path)
        kv = g.kv
        if kv.get("general.architecture") != "qwen35":
            raise ValueError("not a qwen35 model")
        nextn = int(kv.get("qwen35.nextn_predict_layers", 0))
        bc = int(kv["qwen35.block_count"])
        hp = self.hp = HParams(
            n_layer=bc - nextn, n_embd=int(kv["qwen35.embedding_length"]), n_ff=int(kv["qwen35.feed_forward_length"]),
            n_vocab=0, n_head=int(kv["qwen35.attention.head_count"]), n_head_kv=int(kv["qwen35.attention.head_count_kv"]),
            head_dim=int(kv["qwen35.attention.key_length"]), n_rot=int(kv["qwen35.rope.dimension_count"]),
            rope_base=float(np.float32(kv.get("qwen35.rope.freq_base", 10000.0))),
            eps=float(np.float32(kv.get("qwen35.attention.layer_norm_rms_epsilon", 1e-6))),
            conv_k=int(kv["qwen35.ssm.conv_kernel"]), d_inner=int(kv["qwen35.ssm.inner_size"]),
            s_k=int(kv["qwen35.ssm.state_size"]), h_k=int(kv["qwen35.ssm.group_count"]),
            h_v=int(kv["qwen35.ssm.time_step_rank"]))
        interval = int(kv.get("qwen35.full_attention_interval", 4))
        rec = kv.get("qwen35.attention.recurrent_layers")
        self.recurrent = [bool(rec[i]) if rec is not None else (i + 1) % interval != 0 for i in range(hp.n_layer)]
        W = lambda n: Weight(g, g.tensors[n]) if n in g.tensors else None
        self.tok_embd = W("token_embd.weight")
        self.output_norm = W("output_norm.weight")
        self.output = W("output.weight") or self.tok_embd
        toks = kv.get("tokenizer.ggml.tokens")
        hp.n_vocab = len(toks) if toks is not None else self.tok_embd.ne1
        self.layers = []
        for i in range(hp.n_layer + (1 if nextn else 0)):
            P = f"blk.{i}."
            names = [k[len(P):] for k in g.tensors if k.startswith(P)]
            self.layers.append({n.replace(".weight", "").replace(".bias", ""): W(P + n) for n in names})
        self.has_mtp = nextn > 0
        if self.has_mtp:
            L = self.layers[hp.n_layer]
            self.mtp_eh, self.mtp_enorm = L["nextn.eh_proj"], L["nextn.enorm"]
            self.mtp_hnorm, self.mtp_head_norm = L["nextn.hnorm"], L["nextn.shared_head_norm"]

    def embed(self, tok: int) -> np.ndarray:
        """xj_embed (core/xj_cpu.c:369-373): out-of-range ids give zeros."""
        if tok < 0 or tok >= self.tok_embd.ne1:
            return np.zeros(self.hp.n_embd, np.float32)
        return self.tok_embd.row(int(tok))


# ---------------------------------------------------------------- math (xj_cpu.c)
def matmul(w: Weight, x: np.ndarray) -> np.ndarray:
    """y[t][r] = dot(W[r], x[t]) with W dequantised to fp32 (core/xj_cpu.c:36-54)."""
    return (x.astype(np.float32) @ w.f32.T).astype(np.float32)


def rmsnorm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """x * w / sqrt(mean(x^2) + eps), sum in double (core/xj_cpu.c:56-61). Rows along the last axis."""
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    sc = (np.float32(1.0) / np.sqrt((ss / x.shape[-1]).astype(np.float32) + np.float32(eps))).astype(np.float32)
    y = x * sc
    return (y * w if w is not None else y).astype(np.float32)


def l2norm(x: np.ndarray, eps: float) -> np.ndarray:
    """x / sqrt(sum(x^2) + eps) per row, sum in double, multiply by the reciprocal (core/xj_cpu.c:185-193)."""
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    return (x * (np.float32(1.0) / np.sqrt(ss + np.float32(eps)))).astype(np.float32)


def silu(x):
    return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def sigm(x):
    return (np.float32(1) / (np.float32(1) + np.exp(-x))).astype(np.float32)


def softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)


def gdn_token(q, k, v, beta, alpha, z, dt, A, nw, ssm, Hk: int, Hv: int, S: int, eps: float, qscale):
    """One token of the Gated DeltaNet recurrence in float32, as core/xj_cpu.c:194-219 writes it:
    q [Hk][S], k [Hk][S], v [Hv][S] after the convolution; ssm [Hv][S(value j)][S(key i)] updated in place.
    Returns the gated-normalised output [Hv*S]."""
    o = np.zeros(Hv * S, np.float32)
    q = l2norm(q, eps)
    k = l2norm(k, eps)
    b = sigm(beta)
    g = (softplus(alpha + dt) * A).astype(np.float32)
    eg = np.exp(g).astype(np.float32)
    for hv in range(Hv):
        hk = hv % Hk
        M = ssm[hv]                                    # [S(value j)][S(key i)]
        M *= eg[hv]
        sk = M @ k[hk]
        delta = ((v[hv] - sk) * b[hv]).astype(np.float32)
        M += np.outer(delta, k[hk]).astype(np.float32)
        oh = (M @ q[hk]).astype(np.float32) * qscale
        zh = z[hv * S:(hv + 1) * S]
        o[hv * S:(hv + 1) * S] = rmsnorm(oh, nw, eps) * silu(zh)
    return o


def gdn_recurrence(qkv, z, beta, alpha, dt, A, nw, M, Hk: int, Hv: int, S: int, eps: float,
                   dtype=np.float64):
    """The Gated DeltaNet recurrence of attn_linear after its projections and convolution
    (core/xj_cpu.c:194-219), vectorised over value heads, for T tokens of one sequence:
    q, k L2-normalised per key head; b = sigmoid(beta); g = softplus(alpha + dt) * A; per value head
    hv (key head hv % Hk): M *= exp(g); delta = (v - M k) * b; M += delta k^T; o = M q / sqrt(S);
    out = rmsnorm(o) * nw * silu(z). qkv [T][2*Hk*S + Hv*S], z [T][Hv*S], beta/alpha [T][Hv],
    M [Hv][S(value)][S(key)] updated in place. Computed in `dtype` (float64 by default, a tighter
    reference than the float32 of the C code). Returns out [T][Hv*S] as float32."""
    T = qkv.shape[0]
    kd = Hk * S
    hk_of = np.arange(Hv) % Hk
    Md = M.astype(dtype)
    out = np.zeros((T, Hv * S), np.float32)
    qscale = 1.0 / np.sqrt(dtype(S))
    for t in range(T):
        x = qkv[t].astype(dtype)
        q = x[:kd].reshape(Hk, S)
        k = x[kd:2 * kd].reshape(Hk, S)
        v = x[2 * kd:].reshape(Hv, S)
        q = q / np.sqrt((q * q).sum(axis=1, keepdims=True) + eps)
        k = k / np.sqrt((k * k).sum(axis=1, keepdims=True) + eps)
        b = 1.0 / (1.0 + np.exp(-beta[t].astype(dtype)))
        g = np.logaddexp(0.0, alpha[t].astype(dtype) + dt) * A
        kh, qh = k[hk_of], q[hk_of]                                   # [Hv][S]
        Md *= np.exp(g)[:, None, None]
        sk = np.einsum("hji,hi->hj", Md, kh)
        delta = (v - sk) * b[:, None]
        Md += delta[:, :, None] * kh[:, None, :]
        o = np.einsum("hji,hi->hj", Md, qh) * qscale                  # [Hv][S]
        ms = (o * o).mean(axis=1, keepdims=True)
        zz = z[t].astype(dtype).reshape(Hv, S)
        out[t] = (o / np.sqrt(ms + eps) * nw * (zz / (1.0 + np.exp(-zz)))).reshape(-1)
    M[...] = Md
    return out


def rope(v: np.ndarray, n_rot: int, pos: int, base: float) -> np.ndarray:
    """NeoX rotation of the first n_rot dims, pairs (i, i + n_rot/2) (core/xj_cpu.c:68-77)."""
    half = n_rot // 2
    i = np.arange(half, dtype=np.float32)
    theta = (np.float32(pos) * np.power(np.float32(base), np.float32(-2.0) * i / np.float32(n_rot))).astype(np.float32)
    c, s = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
    out = v.astype(np.float32).copy()
    x0, x1 = v[..., :half], v[..., half:n_rot]
    out[..., :half] = x0 * c - x1 * s
    out[..., half:n_rot] = x0 * s + x1 * c
    return out


class Stage:
    """CPU stage over layers [l0, l1) with the reference's state machine (core/xj_cpu.c:228-418).

    forward(x[T][E]) -> x after the layers; logits(x) -> [T][V]; keep / rollback / reset as the
    reference. The KV cache is float32 (the reference CPU cache, core/xj_cpu.c:114-115).
    """

    def __init__(self, m: Model, l0: int, l1: int, n_ctx: int = 256, max_batch: int = 16, has_head: bool = True):
        hp = m.hp
        self.m, self.hp, self.l0, self.l1 = m, hp, l0, l1
        self.mtp = m.has_mtp and l0 == hp.n_layer and l1 == hp.n_layer + 1
        if l0 < 0 or (l1 > hp.n_layer and not self.mtp) or l0 > l1:
            raise ValueError(f"bad layer range [{l0},{l1})")
        self.n_ctx, self.max_batch, self.has_head = n_ctx, max_batch, has_head
        self.n_past, self.keep, self.ck_start, self.ck_T = 0, 0, 0, 0
        self.st = {}
        for il in range(l0, l1):
            if il < hp.n_layer and m.recurrent[il]:
                self.st[il] = dict(conv=np.zeros((hp.conv_dim, hp.conv_k - 1), np.float32),
                                   ssm=np.zeros((hp.h_v, hp.s_v, hp.s_k), np.float32), ck=[])
            else:
                kvd = hp.n_head_kv * hp.head_dim
                self.st[il] = dict(kc=np.zeros((n_ctx, kvd), np.float32), vc=np.zeros((n_ctx, kvd), np.float32))

    def _rec(self, il):
        return il < self.hp.n_layer and self.m.recurrent[il]

    # gated full attention (core/xj_cpu.c:83-151)
    def attn_full(self, il, h, T):
        hp, L, st = self.hp, self.m.layers[il], self.st[il]
        D, H, Hkv = hp.head_dim, hp.n_head, hp.n_head_kv
        nq, nk = 2 * H * D, Hkv * D
        if "attn_qkv" in L:
            qkv = matmul(L["attn_qkv"], h)
            qg, k, v = qkv[:, :nq], qkv[:, nq:nq + nk].copy(), qkv[:, nq + nk:]
        else:
            qg, k, v = matmul(L["attn_q"], h), matmul(L["attn_k"], h), matmul(L["attn_v"], h)
        kn, qn = L["attn_k_norm"].f32[0], L["attn_q_norm"].f32[0]
        for t in range(T):
            pos = self.n_past + t
            kt = k[t].reshape(Hkv, D)
            kt = rope(rmsnorm(kt, kn, hp.eps), hp.n_rot, pos, hp.rope_base)
            st["kc"][pos] = kt.reshape(-1)
            st["vc"][pos] = v[t]
        att = np.zeros((T, H * D), np.float32)
        scale = np.float32(1.0 / np.sqrt(np.float32(D)))
        grp = H // Hkv
        for t in range(T):
            pos = self.n_past + t
            for hh in range(H):
                kvh = hh // grp
                qr = qg[t, hh * 2 * D: hh * 2 * D + D]
                gate = qg[t, hh * 2 * D + D: hh * 2 * D + 2 * D]
                q = rope(rmsnorm(qr, qn, hp.eps), hp.n_rot, pos, hp.rope_base)
                K = st["kc"][:pos + 1, kvh * D:(kvh + 1) * D]
                V = st["vc"][:pos + 1, kvh * D:(kvh + 1) * D]
                sc = (K @ q).astype(np.float32) * scale
                mx = sc.max()
                e = np.exp(sc - mx).astype(np.float32)
                p = (e / e.astype(np.float64).sum()).astype(np.float32)
                o = (p @ V).astype(np.float32)
                att[t, hh * D:(hh + 1) * D] = o * sigm(gate)
        return matmul(L["attn_output"], att)

    # Gated DeltaNet (core/xj_cpu.c:155-223)
    def attn_linear(self, il, h, T):
        hp, L, st = self.hp, self.m.layers[il], self.st[il]
        CD, KC, Hv, Hk, S = hp.conv_dim, hp.conv_k, hp.h_v, hp.h_k, hp.s_k
        qkv = matmul(L["attn_qkv"], h)
        z = matmul(L["attn_gate"], h)
        beta = matmul(L["ssm_beta"], h)
        alpha = matmul(L["ssm_alpha"], h)
        cw = L["ssm_conv1d"].f32          # [CD][KC]
        dt = L["ssm_dt"].f32[0]
        A = L["ssm_a"].f32[0]
        nw = L["ssm_norm"].f32[0]
        qscale = np.float32(1.0 / np.sqrt(np.float32(S)))
        o = np.zeros((T, hp.d_inner), np.float32)
        ck = self.keep and T > 0
        for t in range(T):
            x = qkv[t]
            win = np.concatenate([st["conv"], x[:, None]], axis=1)   # [CD][KC]
            acc = (win * cw).sum(axis=1, dtype=np.float32)
            st["conv"] = win[:, 1:].copy()
            x = silu(acc.astype(np.float32))
            q = x[:hp.key_dim].reshape(Hk, S)
            k = x[hp.key_dim:2 * hp.key_dim].reshape(Hk, S)
            v = x[2 * hp.key_dim:].reshape(Hv, S)
            o[t] = gdn_token(q, k, v, beta[t], alpha[t], z[t], dt, A, nw, st["ssm"], Hk, Hv, S, hp.eps, qscale)
            if ck and t < T - 1:
                st["ck"].append((st["conv"].copy(), st["ssm"].copy()))
        return matmul(L["ssm_out"], o)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """core/xj_cpu.c:244-280."""
        hp = self.hp
        E = hp.n_embd
        x = np.array(x, dtype=np.float32, copy=True)
        T = x.shape[0]
        if T <= 0 or T > self.max_batch:
            self.keep = 0
            raise ValueError(f"T={T} exceeds max_batch {self.max_batch}")
        if self.n_past + T > self.n_ctx:
            self.keep = 0
            raise ValueError(f"context full ({self.n_ctx})")
        for il in self.st:
            if "ck" in self.st[il]:
                self.st[il]["ck"] = []
        self.ck_start = self.n_past
        self.ck_T = T if self.keep else 0
        if self.mtp:
            m = self.m
            hcat = np.concatenate([rmsnorm(x[:, :E], m.mtp_enorm.f32[0], hp.eps),
                                   rmsnorm(x[:, E:2 * E], m.mtp_hnorm.f32[0], hp.eps)], axis=1)
            x = matmul(m.mtp_eh, hcat)
        for il in range(self.l0, self.l1):
            L = self.m.layers[il]
            h = rmsnorm(x, L["attn_norm"].f32[0], hp.eps)
            u = self.attn_linear(il, h, T) if self._rec(il) else self.attn_full(il, h, T)
            x = (x + u).astype(np.float32)
            h = rmsnorm(x, L["post_attention_norm"].f32[0], hp.eps)
            g = matmul(L["ffn_gate"], h)
            a = matmul(L["ffn_up"], h)
            x = (x + matmul(L["ffn_down"], (silu(g) * a).astype(np.float32))).astype(np.float32)
        self.n_past += T
        self.keep = 0
        return x

    def logits(self, x: np.ndarray) -> np.ndarray:
        """core/xj_cpu.c:282-291."""
        if not self.has_head:
            raise ValueError("stage has no output head")
        nw = self.m.mtp_head_norm if self.mtp else self.m.output_norm
        return matmul(self.m.output, rmsnorm(np.asarray(x, np.float32), nw.f32[0], self.hp.eps))

    def rollback(self, n_past: int) -> None:
        """core/xj_cpu.c:293-319."""
        if n_past == self.n_past:
            self.ck_T = 0
            return
        recurrent = any("ssm" in s for s in self.st.values())
        if not recurrent:
            if n_past < 0 or n_past > self.n_past:
                raise ValueError(f"cannot roll back to {n_past}")
            self.n_past = n_past
            return
        j = n_past - self.ck_start - 1
        if not self.ck_T or self.n_past != self.ck_start + self.ck_T or j < 0 or j >= self.ck_T - 1:
            raise ValueError(f"cannot roll back to {n_past}")
        for s in self.st.values():
            if "ssm" in s:
                s["conv"], s["ssm"] = s["ck"][j][0].copy(), s["ck"][j][1].copy()
        self.n_past = n_past
        self.ck_T = 0

    def reset(self) -> None:
        """core/xj_cpu.c:321-330 (the KV cache is not cleared; n_past = 0 makes it unreachable)."""
        for s in self.st.values():
            if "ssm" in s:
                s["conv"][:] = 0
                s["ssm"][:] = 0
        self.n_past = 0


def argmax(x: np.ndarray) -> int:
    """Greedy pick, lowest index on ties (core/xj_spec.c:12-16)."""
    return int(np.argmax(x))


def greedy(m: Model, prompt, n_gen: int, max_batch: int = 8, n_ctx: int = 4096):
    """Greedy decode loop of tools/xjpipe-run.c:24-60 (prefill in chunks, then one token per step)."""
    E = m.hp.n_embd
    s = Stage(m, 0, m.hp.n_layer, n_ctx, max_batch, True)
    prompt = list(prompt)
    lg = None
    for i in range(0, len(prompt), max_batch):
        chunk = prompt[i:i + max_batch]
        x = np.stack([m.embed(t) for t in chunk])
        x = s.forward(x)
        if i + len(chunk) == len(prompt):
            lg = s.logits(x[-1:])[0]
    out = []
    for g in range(n_gen):
        t = argmax(lg)
        out.append(t)
        if g + 1 == n_gen:
            break
        x = s.forward(m.embed(t)[None, :])
        lg = s.logits(x)[0]
    return np.array(out, np.int32)


# ---------------------------------------------------------------- sampling (session layer)
def splitmix64(z: int) -> int:
    """SplitMix64 output function (Steele, Lea and Flood, OOPSLA 2014) on a 64-bit state value."""
    M = (1 << 64) - 1
    z &= M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def sample_uniform(seed: int, counter: int) -> float:
    """The device sampler's draw: 30 bits of splitmix64(seed + (counter + 1) * golden gamma), times 2^-30
    (the resolution of arc4random_uniform(1 << 30) / 2^30 in ios/App/XJGlue.c:279)."""
    z = splitmix64((seed + (counter + 1) * 0x9E3779B97F4A7C15) & ((1 << 64) - 1))
    return (z >> 34) / float(1 << 30)


def sample(lg: np.ndarray, temp: float, u: float, top_k: int = 40, top_p: float = 0.95) -> int:
    """The session layer's sampler (ios/App/XJGlue.c:251-282) with the uniform draw u supplied:
    greedy for temp <= 0; else a running top-k selection (replace the current minimum when a larger
    value arrives), a descending selection sort, p_i = exp((v_i - v_0) / temp) in double, the cut where
    the normalised cumulative sum reaches top_p, r = u * (sum of kept p), first i with r - sum p <= 0."""
    lg = np.asarray(lg, np.float32)
    n = lg.size
    best = int(np.argmax(lg))
    if temp <= 0:
        return best
    K = top_k
    idx, val, k, mi = [0] * K, [0.0] * K, 0, 0
    for i in range(n):
        v = float(lg[i])
        if k < K:
            idx[k], val[k] = i, v
            if v < val[mi]:
                mi = k
            k += 1
        elif v > val[mi]:
            idx[mi], val[mi] = i, v
            mi = min(range(K), key=lambda j: (val[j], j))
    for i in range(k):
        for j in range(i + 1, k):
            if val[j] > val[i]:
                val[i], val[j] = val[j], val[i]
                idx[i], idx[j] = idx[j], idx[i]
    p, s = [], 0.0
    for i in range(k):
        # (val[i] - val[0]) / temp is float arithmetic in the C code; exp takes it as a double
        p.append(float(np.exp(np.float64((np.float32(val[i]) - np.float32(val[0])) / np.float32(temp)))))
        s += p[i]
    acc, cut = 0.0, k
    for i in range(k):
        acc += p[i] / s
        if acc >= top_p:
            cut = i + 1
            break
    s2 = 0.0
    for i in range(cut):
        s2 += p[i]
    r = u * s2
    for i in range(cut):
        r -= p[i]
        if r <= 0:
            return idx[i]
    return idx[0]


def sample_fast(lg: np.ndarray, temp: float, u: float, top_k: int = 40, top_p: float = 0.95) -> int:
    """sample() for rows without equal values at the k-th place, vectorised: the top-k set sorted by value
    descending (index ascending on ties), then the same cut and draw arithmetic."""
    lg = np.asarray(lg, np.float32)
    if temp <= 0:
        return int(np.argmax(lg))
    K = min(top_k, lg.size)
    order = np.lexsort((np.arange(lg.size), -lg.astype(np.float64)))[:K]
    vals = lg[order]
    p, s = [], 0.0
    for i in range(K):
        p.append(float(np.exp(np.float64((vals[i] - vals[0]) / np.float32(temp)))))
        s += p[i]
    acc, cut = 0.0, K
    for i in range(K):
        acc += p[i] / s
        if acc >= top_p:
            cut = i + 1
            break
    s2 = 0.0
    for i in range(cut):
        s2 += p[i]
    r = u * s2
    for i in range(cut):
        r -= p[i]
        if r <= 0:
            return int(order[i])
    return int(order[0])
