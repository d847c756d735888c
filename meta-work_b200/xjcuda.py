"""Python front end of libxj_cuda.so (C ABI in include/xj_cuda.h), used by tests and bench.py.

Everything goes through the library's exported C functions and the xj_stage function pointers the
library fills in, exactly as a C host (or the runtime's own pipeline code) would call them. There is
no Python or CPU fallback: if the library or a GPU is missing, the calls fail.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "csrc" / "libxj_cuda.so"

_lib = None

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30
OPT_KV_F32, OPT_GEMV, OPT_PDL, OPT_PERSIST, OPT_TRACE, OPT_GEMV_CTAS, OPT_TC = 1, 2, 3, 4, 5, 6, 7


class XjError(RuntimeError):
    pass


# ---- ABI mirror of include/xj_abi.h (only what Python touches) ----
FORWARD = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t)
LOGITS = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p,
                          ctypes.c_size_t)
ROLLBACK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t)
VOIDFN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


class _Stage(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_void_p), ("l0", ctypes.c_int), ("l1", ctypes.c_int), ("n_ctx", ctypes.c_int),
        ("max_batch", ctypes.c_int), ("n_past", ctypes.c_int), ("has_head", ctypes.c_bool), ("mtp", ctypes.c_bool),
        ("backend", ctypes.c_char_p), ("keep", ctypes.c_int), ("ck_start", ctypes.c_int), ("ck_T", ctypes.c_int),
        ("forward", FORWARD), ("logits", LOGITS), ("rollback", ROLLBACK), ("reset", VOIDFN), ("destroy", VOIDFN),
        ("impl", ctypes.c_void_p),
    ]


class _HParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n_layer", "n_embd", "n_ff", "n_vocab", "n_head", "n_head_kv", "head_dim",
                                             "n_rot")] + \
               [("rope_base", ctypes.c_float), ("eps", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("conv_k", "d_inner", "s_k", "h_k", "h_v", "s_v", "key_dim", "conv_dim",
                                             "full_attn_interval")] + \
               [("eos", ctypes.c_uint32), ("eot", ctypes.c_uint32)]


class _W(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("file_off", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("type", ctypes.c_uint32), ("ne0", ctypes.c_int64), ("ne1", ctypes.c_int64)]


class _Layer(ctypes.Structure):
    _fields_ = [("recurrent", ctypes.c_bool)] + [(n, _W) for n in (
        "attn_norm", "post_norm", "wqkv", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "ssm_qkv", "ssm_gate",
        "ssm_conv1d", "ssm_dt", "ssm_a", "ssm_beta", "ssm_alpha", "ssm_norm", "ssm_out", "ffn_gate", "ffn_up",
        "ffn_down")]


class _Model(ctypes.Structure):
    _fields_ = [("gguf", ctypes.c_void_p), ("hp", _HParams), ("tok_embd", _W), ("output_norm", _W), ("output", _W),
                ("layers", _Layer * 128), ("fingerprint", ctypes.c_uint64), ("has_mtp", ctypes.c_bool),
                ("mtp_eh", _W), ("mtp_enorm", _W), ("mtp_hnorm", _W), ("mtp_head_norm", _W),
                ("mtp_gguf", ctypes.c_void_p)]


def build(quiet: bool = True) -> None:
    """Compile csrc/libxj_cuda.so (nvcc, sm_100a)."""
    r = subprocess.run(["make", "-C", str(LIB.parent)], capture_output=True, text=True)
    if r.returncode != 0:
        raise XjError("build failed:\n" + r.stdout[-4000:] + r.stderr[-4000:])


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        build()
    L = ctypes.CDLL(str(LIB))
    vp, ip, sz, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p
    sig = {
        "xj_cuda_stage_new": (ctypes.POINTER(_Stage), [vp, ip, ip, ip, ip, ctypes.c_bool, cp, sz]),
        "xj_cuda_device_name": (cp, []),
        "xjc_model_load": (vp, [cp, cp, sz]),
        "xjc_model_free": (None, [vp]),
        "xjc_embed": (None, [vp, ctypes.c_int32, vp]),
        "xjc_stage_state_bytes": (ctypes.c_uint64, [vp, ip, ip, ip, ip]),
        "xj_cuda_set_options": (ip, [ip, ip]),
        "xj_cuda_decode": (ip, [vp, vp, ip, ip, vp, vp, vp, cp, sz]),
        "xj_cuda_dequant_rows": (ip, [ip, vp, ip, ip, vp, cp, sz]),
        "xj_cuda_tc_selftest": (ip, [vp, vp, ip, vp, cp, sz]),
        "xj_cuda_graph_kernels": (ip, [vp]),
        "xj_cuda_last_decode_launches": (ctypes.c_longlong, [vp, vp]),
        "xj_cuda_phase_trace": (ip, [vp, vp, ip]),
        "xj_cuda_batch_new": (vp, [vp, ip, ip, cp, sz]),
        "xj_cuda_batch_free": (None, [vp]),
        "xj_cuda_batch_reset": (ip, [vp, cp, sz]),
        "xj_cuda_batch_n_past": (ip, [vp]),
        "xj_cuda_batch_decode": (ip, [vp, vp, ip, ip, vp, vp, vp, cp, sz]),
        "xj_cuda_batch_last_launches": (ctypes.c_longlong, [vp, vp]),
        "xj_cuda_gemv": (ip, [ip, vp, ip, ip, vp, ip, vp, ip, cp, sz]),
        "xj_cuda_gemv_time": (ip, [ip, vp, ip, ip, ip, ip, ip, ip, vp, cp, sz]),
        "xj_cuda_gdn_time": (ip, [ip, ip, ip, ip, vp, cp, sz]),
        "xj_cuda_spec_decode": (ip, [vp, vp, vp, ip, ip, ip, vp, vp, cp, sz]),
        "xj_cuda_gdn_prefill_check": (ip, [ip, ip, ip, ip, vp, cp, sz]),
        "xj_cuda_norm_gemv_noalloc": (ip, [ip, vp, ip, ip, vp, vp, ctypes.c_float, ip, vp, cp, sz]),
        "xj_cuda_gdn_run": (ip, [ip, ip, ip, ip, ip, vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, vp, vp, cp, sz]),
        "xj_cuda_set_sampler": (ip, [vp, ctypes.c_float, ip, ctypes.c_double, ctypes.c_ulonglong, cp, sz]),
        "xj_cuda_batch_new_multi": (vp, [vp, ip, ip, ip, cp, sz]),
        "xj_cuda_batch_spec_decode": (ip, [vp, vp, vp, ip, ip, ip, vp, vp, vp, cp, sz]),
        "xj_cuda_pipeline_id_new": (ip, [vp, cp, sz]),
        "xj_cuda_pipeline_new": (vp, [vp, ip, ip, vp, ip, ip, ip, cp, sz]),
        "xj_cuda_pipeline_free": (None, [vp]),
        "xj_cuda_pipeline_batch": (vp, [vp]),
        "xj_cuda_pipeline_decode": (ip, [vp, vp, ip, ip, vp, vp, cp, sz]),
        "xj_cuda_sample_logits": (ip, [vp, ip, ip, ctypes.c_float, ip, ctypes.c_double, ctypes.c_ulonglong,
                                       ctypes.c_ulonglong, vp, vp, cp, sz]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def ctor_address() -> int:
    """Address of xj_cuda_stage_new, for hosts that take a stage constructor (same signature as xj_cpu_stage_new)."""
    return ctypes.cast(lib().xj_cuda_stage_new, ctypes.c_void_p).value


def set_option(which: int, value: int) -> None:
    if lib().xj_cuda_set_options(which, value) != 0:
        raise XjError(f"unknown option {which}")


def device_name() -> str:
    return lib().xj_cuda_device_name().decode()


def dequant_rows(type_id: int, raw: bytes, k: int, n_rows: int) -> np.ndarray:
    """GPU block decoder on host bytes -> fp32 [n_rows][k] (xj_cuda_dequant_rows)."""
    src = np.frombuffer(bytes(raw), np.uint8).copy()
    out = np.zeros((n_rows, k), np.float32)
    e = _err()
    if lib().xj_cuda_dequant_rows(type_id, src.ctypes.data, k, n_rows, out.ctypes.data, e, 512):
        _raise(e)
    return out


def tc_selftest(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """d[128][64] = a[128][k] . b[64][k]^T on the tcgen05 tensor cores (a, b float16; xj_cuda_tc_selftest)."""
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    assert a.shape[0] == 128 and b.shape[0] == 64 and a.shape[1] == b.shape[1]
    d = np.zeros((128, 64), np.float32)
    e = _err()
    if lib().xj_cuda_tc_selftest(a.ctypes.data, b.ctypes.data, a.shape[1], d.ctypes.data, e, 512):
        _raise(e)
    return d


def gemv(type_id: int, raw: bytes, k: int, n: int, x: np.ndarray, path: int = 0) -> np.ndarray:
    """y[T][n] = W x with the decode GEMV kernels (xj_cuda_gemv)."""
    w = np.frombuffer(bytes(raw), np.uint8).copy()
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    e = _err()
    if lib().xj_cuda_gemv(type_id, w.ctypes.data, k, n, x.ctypes.data, x.shape[0], y.ctypes.data, path, e, 512):
        _raise(e)
    return y


def gemv_time(type_id: int, raw: bytes, k: int, n: int, T: int = 1, copies: int = 4, iters: int = 50,
              path: int = 0) -> float:
    """Average ms per GEMV launch with weights rotated over `copies` device copies (xj_cuda_gemv_time)."""
    w = np.frombuffer(bytes(raw), np.uint8).copy()
    ms = ctypes.c_float(0)
    e = _err()
    if lib().xj_cuda_gemv_time(type_id, w.ctypes.data, k, n, T, copies, iters, path, ctypes.byref(ms), e, 512):
        _raise(e)
    return ms.value


def gdn_time(S: int, Hv: int, B: int, iters: int = 50) -> float:
    """Average ms per Gated DeltaNet decode step of B sequences x Hv heads (xj_cuda_gdn_time)."""
    ms = ctypes.c_float(0)
    e = _err()
    if lib().xj_cuda_gdn_time(S, Hv, B, iters, ctypes.byref(ms), e, 512):
        _raise(e)
    return ms.value


def gdn_prefill_check(S: int, Hk: int, Hv: int, T: int):
    """Chunked vs token-by-token Gated DeltaNet over T tokens (xj_cuda_gdn_prefill_check):
    (max rel diff of outputs, of the final state, chunked ms, token-by-token ms)."""
    r = np.zeros(4, np.float32)
    e = _err()
    if lib().xj_cuda_gdn_prefill_check(S, Hk, Hv, T, r.ctypes.data, e, 512):
        _raise(e)
    return tuple(float(v) for v in r)


def gdn_run(path: int, S: int, Hk: int, Hv: int, qkv, z, beta, alpha, dt, A, norm_w, state, eps: float = 1e-6):
    """Gated DeltaNet recurrence on host operands (xj_cuda_gdn_run). path 0 = token-by-token kernel,
    1 = chunked prefill kernels, 2 = batch decode kernel (rows = independent sequences). Returns
    (out [T][Hv*S], final state)."""
    f = lambda a: np.ascontiguousarray(a, np.float32)
    qkv, z, beta, alpha, dt, A, norm_w = map(f, (qkv, z, beta, alpha, dt, A, norm_w))
    st = f(state).copy()
    T = qkv.shape[0]
    out = np.zeros((T, Hv * S), np.float32)
    e = _err()
    if lib().xj_cuda_gdn_run(path, S, Hk, Hv, T, qkv.ctypes.data, z.ctypes.data, beta.ctypes.data, alpha.ctypes.data,
                             dt.ctypes.data, A.ctypes.data, norm_w.ctypes.data, eps, st.ctypes.data, out.ctypes.data,
                             e, 512):
        _raise(e)
    return out, st


def sample_logits(logits, temperature: float, seed: int, counter0: int = 0, top_k: int = 40, top_p: float = 0.95):
    """Device top-k / top-p / temperature pick per row of host logits (xj_cuda_sample_logits): row r
    draws with uniform(seed, counter0 + r). Returns (ids, top-2 margins)."""
    lg = np.ascontiguousarray(logits, np.float32)
    if lg.ndim == 1:
        lg = lg[None]
    rows, n = lg.shape
    out = np.zeros(rows, np.int32)
    mar = np.zeros(rows, np.float32)
    e = _err()
    if lib().xj_cuda_sample_logits(lg.ctypes.data, rows, n, temperature, top_k, top_p, seed, counter0, out.ctypes.data,
                                   mar.ctypes.data, e, 512):
        _raise(e)
    return out, mar


def _err():
    return ctypes.create_string_buffer(512)


def _raise(e):
    raise XjError(e.value.decode(errors="replace"))


class Model:
    """A qwen35 GGUF loaded by the library's loader (xjc_model_load), or wrapping a pointer to an xj_model
    produced by any loader with the runtime's layout (e.g. the runtime's own xj_model_load)."""

    def __init__(self, path: str | os.PathLike | None = None, ptr: int | None = None):
        self.owned = ptr is None
        if ptr is None:
            e = _err()
            ptr = lib().xjc_model_load(str(path).encode(), e, 512)
            if not ptr:
                _raise(e)
        self.ptr = ptr
        self.m = _Model.from_address(ptr)
        self.hp = self.m.hp
        self.n_embd, self.n_vocab, self.n_layer = self.hp.n_embd, self.hp.n_vocab, self.hp.n_layer

    def embed(self, tok: int) -> np.ndarray:
        out = np.zeros(self.n_embd, np.float32)
        lib().xjc_embed(self.ptr, int(tok), out.ctypes.data)
        return out

    def embed_many(self, toks) -> np.ndarray:
        return np.stack([self.embed(int(t)) for t in toks])

    def close(self):
        if self.ptr and self.owned:
            lib().xjc_model_free(self.ptr)
        self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Stage:
    """xj_cuda_stage_new(m, l0, l1, n_ctx, max_batch, has_head) and its vtable."""

    def __init__(self, model: Model, l0: int, l1: int, n_ctx: int = 256, max_batch: int = 16, has_head: bool = True):
        e = _err()
        p = lib().xj_cuda_stage_new(model.ptr, l0, l1, n_ctx, max_batch, has_head, e, 512)
        if not p:
            _raise(e)
        self.model, self.p, self.s = model, p, p.contents
        self.E = model.n_embd

    @property
    def addr(self) -> int:
        return ctypes.cast(self.p, ctypes.c_void_p).value

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        T = x.shape[0]
        e = _err()
        if self.s.forward(self.addr, x.ctypes.data, T, e, 512):
            _raise(e)
        return x.reshape(-1)[:T * self.E].reshape(T, self.E).copy()

    def logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.zeros((T, self.model.n_vocab), np.float32)
        e = _err()
        if self.s.logits(self.addr, x.ctypes.data, T, out.ctypes.data, e, 512):
            _raise(e)
        return out

    def rollback(self, n_past: int) -> None:
        e = _err()
        if self.s.rollback(self.addr, n_past, e, 512):
            _raise(e)

    def reset(self) -> None:
        self.s.reset(self.addr)

    @property
    def keep(self) -> int:
        return self.s.keep

    @keep.setter
    def keep(self, v: int) -> None:
        self.s.keep = v

    @property
    def n_past(self) -> int:
        return self.s.n_past

    @property
    def ck(self):
        return self.s.ck_start, self.s.ck_T

    @property
    def backend(self) -> str:
        return self.s.backend.decode()

    def decode(self, prompt, n_gen: int, want_margins: bool = False):
        """Device-resident greedy decode (xj_cuda_decode). Returns (ids, margins or None, gpu_ms[2])."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, np.int32)
        mar = np.zeros(n_gen, np.float32) if want_margins else None
        ms = np.zeros(2, np.float32)
        e = _err()
        rc = lib().xj_cuda_decode(self.addr, p.ctypes.data, p.size, n_gen, out.ctypes.data,
                                  mar.ctypes.data if mar is not None else None, ms.ctypes.data, e, 512)
        if rc:
            _raise(e)
        return out, mar, ms

    def set_sampler(self, temperature: float, seed: int = 0, top_k: int = 40, top_p: float = 0.95) -> None:
        """Sample later decode() tokens (top-k / top-p / temperature, xj_cuda_set_sampler); temperature <= 0
        restores greedy decoding."""
        e = _err()
        if lib().xj_cuda_set_sampler(self.addr, temperature, top_k, top_p, seed, e, 512):
            _raise(e)

    def spec_decode(self, draft: "Stage", prompt, n_gen: int, k: int = 4):
        """Greedy speculative decode with a draft-model stage (xj_cuda_spec_decode). Returns (ids, stats)
        with stats = (target verify forwards, drafted, accepted, draft re-feeds)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, np.int32)
        st = (ctypes.c_longlong * 4)()
        e = _err()
        if lib().xj_cuda_spec_decode(self.addr, draft.addr, p.ctypes.data, p.size, n_gen, k, out.ctypes.data, st, e, 512):
            _raise(e)
        return out, tuple(int(v) for v in st)

    def last_decode_launches(self) -> tuple[int, int]:
        """Kernel launches of the last decode() call: (prompt, decode steps after it); the persistent
        kernel runs up to 8192 steps per launch."""
        v = (ctypes.c_longlong * 2)()
        lib().xj_cuda_last_decode_launches(self.addr, v)
        return int(v[0]), int(v[1])

    def phase_trace(self):
        """Per-phase timing of the last traced persistent decode (OPT_TRACE): array [phases, 13] of
        kind, max CTA us, mean CTA us, span us, start us, mean weight wait us, mean request lead us, then
        for matrix-vector phases the mean prologue us, mean first-tile us, and the first tile's chunk
        wait, tensor-core work, tile barrier and epilogue us; for attention phases the mean us of an
        item's steps (position read, query/key norm, cache rows staged, rounds, split counter) and of
        the split merge."""
        out = np.zeros((4096, 13), np.float64)
        n = lib().xj_cuda_phase_trace(self.addr, out.ctypes.data, 4096)
        if n < 0:
            raise XjError("no phase trace (enable OPT_TRACE before decode)")
        return out[:n]

    def close(self):
        if self.p:
            self.s.destroy(self.addr)
            self.p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """n_seq independent sequences decoded in lockstep on one GPU (xj_cuda_batch_*)."""

    def __init__(self, model: Model, n_seq: int, n_ctx: int = 256, max_tokens: int = 1):
        """max_tokens > 1 (xj_cuda_batch_new_multi): forwards of up to that many tokens per sequence (chunked
        prompts of batches wider than 16 sequences, the target of spec_decode)."""
        e = _err()
        if max_tokens > 1:
            p = lib().xj_cuda_batch_new_multi(model.ptr, n_seq, n_ctx, max_tokens, e, 512)
        else:
            p = lib().xj_cuda_batch_new(model.ptr, n_seq, n_ctx, e, 512)
        if not p:
            _raise(e)
        self.model, self.p, self.n_seq = model, p, n_seq

    @property
    def n_past(self) -> int:
        return int(lib().xj_cuda_batch_n_past(self.p))

    def reset(self):
        e = _err()
        if lib().xj_cuda_batch_reset(self.p, e, 512):
            _raise(e)

    def decode(self, prompts, n_gen: int, want_margins: bool = False):
        """prompts [n_seq][n_prompt] -> (ids [n_seq][n_gen], margins or None, gpu_ms[2])."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        assert p.ndim == 2 and p.shape[0] == self.n_seq
        out = np.zeros((self.n_seq, n_gen), np.int32)
        mar = np.zeros((self.n_seq, n_gen), np.float32) if want_margins else None
        ms = np.zeros(2, np.float32)
        e = _err()
        rc = lib().xj_cuda_batch_decode(self.p, p.ctypes.data, p.shape[1], n_gen, out.ctypes.data,
                                        mar.ctypes.data if mar is not None else None, ms.ctypes.data, e, 512)
        if rc:
            _raise(e)
        return out, mar, ms

    def spec_decode(self, draft: "Batch", prompts, n_gen: int, k: int = 4):
        """Greedy speculative decoding of every sequence with a draft batch (xj_cuda_batch_spec_decode).
        Returns (ids [n_seq][n_gen], stats (rounds, drafted, accepted, target rows), device ms)."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        assert p.ndim == 2 and p.shape[0] == self.n_seq
        out = np.zeros((self.n_seq, n_gen), np.int32)
        st = (ctypes.c_longlong * 4)()
        ms = ctypes.c_float(0)
        e = _err()
        if lib().xj_cuda_batch_spec_decode(self.p, draft.p, p.ctypes.data, p.shape[1], n_gen, k, out.ctypes.data, st,
                                           ctypes.byref(ms), e, 512):
            _raise(e)
        return out, tuple(int(v) for v in st), ms.value

    def last_launches(self) -> tuple[int, int]:
        v = (ctypes.c_longlong * 2)()
        lib().xj_cuda_batch_last_launches(self.p, v)
        return int(v[0]), int(v[1])

    def close(self):
        if self.p:
            lib().xj_cuda_batch_free(self.p)
            self.p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


PIPELINE_ID_BYTES = 384


def pipeline_id() -> bytes:
    """A new identifier for the communicators of one pipeline (xj_cuda_pipeline_id_new), made on rank 0 and
    handed to every rank by the host (any channel: a store, a pipe, a file)."""
    buf = (ctypes.c_ubyte * PIPELINE_ID_BYTES)()
    e = _err()
    if lib().xj_cuda_pipeline_id_new(buf, e, 512):
        _raise(e)
    return bytes(buf)


class Pipeline:
    """This rank's part of a layer pipeline across GPUs over NCCL (xj_cuda_pipeline_*): layers split evenly
    over the world's ranks, n_seq sequences in n_micro micro-batches. Collective: every rank constructs it
    (on its own current device) and calls decode together."""

    def __init__(self, model: Model, rank: int, world: int, pid: bytes | None, n_seq: int, n_ctx: int = 256,
                 n_micro: int = 2):
        e = _err()
        idb = (ctypes.c_ubyte * PIPELINE_ID_BYTES).from_buffer_copy(pid) if pid is not None else None
        p = lib().xj_cuda_pipeline_new(model.ptr, rank, world, idb, n_seq, n_ctx, n_micro, e, 512)
        if not p:
            _raise(e)
        self.p, self.rank, self.world, self.n_seq, self.model = p, rank, world, n_seq, model

    def decode(self, prompts, n_gen: int):
        """Rank 0: prompts [n_seq][n_prompt] -> (ids [n_seq][n_gen], device ms); other ranks pass the
        prompt length as an int and get (None, device ms)."""
        ms = ctypes.c_float(0)
        e = _err()
        if self.rank == 0:
            pr = np.ascontiguousarray(prompts, dtype=np.int32)
            assert pr.ndim == 2 and pr.shape[0] == self.n_seq
            out = np.zeros((self.n_seq, n_gen), np.int32)
            rc = lib().xj_cuda_pipeline_decode(self.p, pr.ctypes.data, pr.shape[1], n_gen, out.ctypes.data,
                                               ctypes.byref(ms), e, 512)
        else:
            out = None
            rc = lib().xj_cuda_pipeline_decode(self.p, None, int(prompts), n_gen, None, ctypes.byref(ms), e, 512)
        if rc:
            _raise(e)
        return out, ms.value

    def close(self):
        if self.p:
            lib().xj_cuda_pipeline_free(self.p)
            self.p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
