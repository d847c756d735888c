"""ctypes front end of oracle/_ref/libxjref.so: the reference CPU path of xiaoju-pipe.

TEST INFRASTRUCTURE ONLY. The library is the reference's own core/*.c built unchanged by
oracle/Makefile plus oracle/ref_harness.c. tests/, __graft_entry__.smoke() and bench.py's CPU legs use
it as the checker / the timed CPU baseline; the CUDA product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libxjref.so"
# the reference source tree (read-only): $XJ_REF_TREE, else the checkout location of this build machine
REF_TREE = pathlib.Path(os.environ.get("XJ_REF_TREE", "/root/reference/src/xiaoju-pipe"))

_lib = None

c_float_p = ctypes.POINTER(ctypes.c_float)
c_i32_p = ctypes.POINTER(ctypes.c_int32)


def build() -> bool:
    """Build _ref/libxjref.so when the reference tree is present; True when the library exists."""
    if REF_TREE.exists():
        subprocess.run(["make", "-C", str(HERE), f"REF={REF_TREE}"], check=True, capture_output=True)
    return LIB.exists()


def available() -> bool:
    return LIB.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists() and not build():
        raise FileNotFoundError(f"{LIB} missing (build it with `make -C oracle` where the reference tree exists)")
    L = ctypes.CDLL(str(LIB))
    vp, ip, fp = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    sig = {
        "xjr_abi": (ip, [ip]),
        "xjr_threads": (ip, []),
        "xjr_set_threads": (None, [ip]),
        "xjr_f16": (fp, [ctypes.c_uint16]),
        "xjr_to_f16": (ctypes.c_uint16, [fp]),
        "xjr_dequant_row": (None, [ctypes.c_uint32, vp, vp, ctypes.c_int64]),
        "xjr_row_bytes": (ctypes.c_uint64, [ctypes.c_uint32, ctypes.c_int64]),
        "xjr_load": (vp, [ctypes.c_char_p, ctypes.c_char_p, ip]),
        "xjr_model_free": (None, [vp]),
        "xjr_n_vocab": (ip, [vp]),
        "xjr_n_embd": (ip, [vp]),
        "xjr_n_layer": (ip, [vp]),
        "xjr_has_mtp": (ip, [vp]),
        "xjr_fingerprint": (ctypes.c_uint64, [vp]),
        "xjr_embed": (None, [vp, ctypes.c_int32, vp]),
        "xjr_attach_mtp": (ip, [vp, ctypes.c_char_p, ctypes.c_char_p, ip]),
        "xjr_stage_new_with": (vp, [vp, vp, ip, ip, ip, ip, ip, ctypes.c_char_p, ip]),
        "xjr_forward": (ip, [vp, vp, ip, ctypes.c_char_p, ip]),
        "xjr_logits": (ip, [vp, vp, ip, vp, ctypes.c_char_p, ip]),
        "xjr_rollback": (ip, [vp, ip, ctypes.c_char_p, ip]),
        "xjr_reset": (None, [vp]),
        "xjr_destroy": (None, [vp]),
        "xjr_set_keep": (None, [vp, ip]),
        "xjr_n_past": (ip, [vp]),
        "xjr_ck": (ip, [vp, ip]),
        "xjr_backend": (ctypes.c_char_p, [vp]),
        "xjr_state_bytes": (ctypes.c_uint64, [vp, ip, ip, ip, ip]),
        "xjr_greedy_with": (ip, [vp, vp, vp, ip, ip, ip, ip, vp, vp, vp, vp, ctypes.c_char_p, ip]),
        "xjr_layer_trace_with": (ip, [vp, vp, vp, vp, ip, ip, ip, vp, vp, ctypes.c_char_p, ip]),
        "xjr_spec_with": (ip, [vp, vp, vp, ip, ip, ip, ip, ip, ip, vp, ip, ip, vp, vp, ctypes.c_char_p, ip]),
        "xjr_eos": (ip, [vp, ip]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class RefError(RuntimeError):
    pass


def _err():
    return ctypes.create_string_buffer(512)


def dequant_row(type_id: int, raw: bytes | np.ndarray, n: int) -> np.ndarray:
    """The reference's xj_dequant_row (core/xj_quant.h:55-122) on one row of n elements."""
    src = np.frombuffer(bytes(raw), dtype=np.uint8).copy()
    out = np.zeros(n, dtype=np.float32)
    lib().xjr_dequant_row(type_id, _ptr(src), _ptr(out), n)
    return out


def row_bytes(type_id: int, n: int) -> int:
    return int(lib().xjr_row_bytes(type_id, n))


def f16_to_f32(h: int) -> float:
    return float(lib().xjr_f16(h))


def f32_to_f16(f: float) -> int:
    return int(lib().xjr_to_f16(f))


def set_threads(n: int) -> None:
    lib().xjr_set_threads(n)


def threads() -> int:
    return int(lib().xjr_threads())


class Model:
    """A model loaded by the reference's own loader, xj_model_load (core/xj_model.c:204-210)."""

    def __init__(self, path: str | os.PathLike):
        e = _err()
        self.ptr = lib().xjr_load(str(path).encode(), e, 512)
        if not self.ptr:
            raise RefError(e.value.decode(errors="replace"))
        self.n_vocab = lib().xjr_n_vocab(self.ptr)
        self.n_embd = lib().xjr_n_embd(self.ptr)
        self.n_layer = lib().xjr_n_layer(self.ptr)
        self.path = str(path)

    @property
    def has_mtp(self) -> bool:
        return bool(lib().xjr_has_mtp(self.ptr))

    @property
    def fingerprint(self) -> int:
        return int(lib().xjr_fingerprint(self.ptr))

    def eos(self) -> tuple[int, int]:
        return lib().xjr_eos(self.ptr, 0), lib().xjr_eos(self.ptr, 1)

    def embed(self, tok: int) -> np.ndarray:
        out = np.zeros(self.n_embd, dtype=np.float32)
        lib().xjr_embed(self.ptr, tok, _ptr(out))
        return out

    def embed_many(self, toks) -> np.ndarray:
        return np.stack([self.embed(int(t)) for t in toks])

    def close(self):
        if self.ptr:
            lib().xjr_model_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- whole-loop helpers ----
    def greedy(self, prompt, n_gen: int, max_batch: int = 8, n_ctx: int = 4096, ctor: int | None = None):
        """Greedy decode (tools/xjpipe-run.c:24-60 pattern). Returns (tokens, margins, first_logits, times)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        tok = np.zeros(n_gen, dtype=np.int32)
        mar = np.zeros(n_gen, dtype=np.float32)
        first = np.zeros(self.n_vocab, dtype=np.float32)
        times = np.zeros(2, dtype=np.float64)
        e = _err()
        rc = lib().xjr_greedy_with(ctor, self.ptr, _ptr(p), p.size, n_gen, max_batch, n_ctx, _ptr(tok), _ptr(mar),
                                   _ptr(first), _ptr(times), e, 512)
        if rc:
            raise RefError(e.value.decode(errors="replace"))
        return tok, mar, first, times

    def layer_trace(self, toks, chunks, max_batch: int = 16, n_ctx: int = 256, ctor: int | None = None):
        """Activations after every layer for the last chunk: hid[L+1][T][E] and logits[T][V]."""
        t = np.ascontiguousarray(toks, dtype=np.int32)
        c = np.ascontiguousarray(chunks, dtype=np.int32)
        T = int(c[-1])
        hid = np.zeros((self.n_layer + 1, T, self.n_embd), dtype=np.float32)
        lg = np.zeros((T, self.n_vocab), dtype=np.float32)
        e = _err()
        rc = lib().xjr_layer_trace_with(ctor, self.ptr, _ptr(t), _ptr(c), c.size, max_batch, n_ctx, _ptr(hid),
                                        _ptr(lg), e, 512)
        if rc:
            raise RefError(e.value.decode(errors="replace"))
        return hid, lg

    def spec(self, prompt, n_gen: int, k: int, max_batch: int = 8, n_ctx: int = 1024, s1: int = 0,
             oracle=None, oracle_miss: int = 0, ctor: int | None = None):
        """Reference pipeline + MTP speculative loop (core/xj_spec.c). Returns (tokens, stats[4])."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        o = np.ascontiguousarray(oracle if oracle is not None else [], dtype=np.int32)
        out = np.zeros(n_gen, dtype=np.int32)
        st = np.zeros(4, dtype=np.float64)
        e = _err()
        n = lib().xjr_spec_with(ctor, self.ptr, _ptr(p), p.size, n_gen, max_batch, n_ctx, s1, k,
                                _ptr(o) if o.size else None, o.size, oracle_miss, _ptr(out), _ptr(st), e, 512)
        if n < 0:
            raise RefError(e.value.decode(errors="replace"))
        return out[:n], st


class Stage:
    """One reference stage (any backend constructor with the xj_cpu_stage_new signature)."""

    def __init__(self, model: Model, l0: int, l1: int, n_ctx: int = 256, max_batch: int = 16,
                 has_head: bool = True, ctor: int | None = None):
        e = _err()
        self.model = model
        self.ptr = lib().xjr_stage_new_with(ctor, model.ptr, l0, l1, n_ctx, max_batch, int(has_head), e, 512)
        if not self.ptr:
            raise RefError(e.value.decode(errors="replace"))
        self.E = model.n_embd

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        T = x.shape[0]
        e = _err()
        if lib().xjr_forward(self.ptr, _ptr(x), T, e, 512):
            raise RefError(e.value.decode(errors="replace"))
        # an MTP stage takes [T][2E] and writes its [T][E] result to the first T*E floats
        return x.reshape(-1)[:T * self.E].reshape(T, self.E).copy()

    def logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.zeros((T, self.model.n_vocab), dtype=np.float32)
        e = _err()
        if lib().xjr_logits(self.ptr, _ptr(x), T, _ptr(out), e, 512):
            raise RefError(e.value.decode(errors="replace"))
        return out

    def rollback(self, n_past: int) -> None:
        e = _err()
        if lib().xjr_rollback(self.ptr, n_past, e, 512):
            raise RefError(e.value.decode(errors="replace"))

    def reset(self):
        lib().xjr_reset(self.ptr)

    @property
    def keep(self):
        raise AttributeError

    @keep.setter
    def keep(self, v: int):
        lib().xjr_set_keep(self.ptr, v)

    @property
    def n_past(self) -> int:
        return lib().xjr_n_past(self.ptr)

    @property
    def ck(self) -> tuple[int, int]:
        return lib().xjr_ck(self.ptr, 0), lib().xjr_ck(self.ptr, 1)

    @property
    def backend(self) -> str:
        return lib().xjr_backend(self.ptr).decode()

    def close(self):
        if self.ptr:
            lib().xjr_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
