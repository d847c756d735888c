"""ctypes front end of the reference's session layer (ios/App/XJGlue.c: the C API its Swift app calls),
built unmodified by oracle/Makefile into oracle/_ref/libxjglue_cpu.so (CPU stages, as the reference
builds it on Linux) and oracle/_ref/libxjglue_cuda.so (its stage constructor taken from libxj_cuda.so).

TEST INFRASTRUCTURE ONLY: tests drive the exact entry points Swift calls (xjg_host_new, xjg_host_chat,
xjg_host_reset, xjg_host_free; XJGlue.h:25-68) over both builds and compare the answers.
"""
from __future__ import annotations

import ctypes
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
LIBS = {"cpu": HERE / "_ref" / "libxjglue_cpu.so", "cuda": HERE / "_ref" / "libxjglue_cuda.so"}
PIECE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int)


class Stats(ctypes.Structure):
    """xjg_stats (XJGlue.h:38-47)."""
    _fields_ = [("prompt_tokens", ctypes.c_int), ("gen_tokens", ctypes.c_int), ("prefill_s", ctypes.c_double),
                ("gen_s", ctypes.c_double), ("local_ms", ctypes.c_double), ("remote_ms", ctypes.c_double),
                ("wait_ms", ctypes.c_double), ("n_past", ctypes.c_int), ("n_ctx", ctypes.c_int),
                ("reconnects", ctypes.c_int), ("spec_steps", ctypes.c_int), ("spec_drafted", ctypes.c_int),
                ("spec_accepted", ctypes.c_int), ("draft_ms", ctypes.c_double)]


def available(which: str) -> bool:
    return LIBS[which].exists()


def lib(which: str) -> ctypes.CDLL:
    L = ctypes.CDLL(str(LIBS[which]))
    vp, ip, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
    L.xjg_host_new.restype = vp
    L.xjg_host_new.argtypes = [cp, cp, ip, ctypes.c_uint32, ip, ip, ip, cp, ip, cp, ip, cp, ip]
    L.xjg_host_chat.restype = ip
    L.xjg_host_chat.argtypes = [vp, cp, ctypes.c_float, ip, PIECE, vp, ctypes.POINTER(Stats), cp, ip]
    L.xjg_host_reset.restype = ip
    L.xjg_host_reset.argtypes = [vp, cp, ip]
    L.xjg_host_free.restype = None
    L.xjg_host_free.argtypes = [vp]
    L.xjg_worker_new.restype = vp
    L.xjg_worker_new.argtypes = [cp, ip, ip, ctypes.c_uint32, vp, vp, cp, ip]
    L.xjg_worker_run.restype = ip
    L.xjg_worker_run.argtypes = [vp, ip, cp, ip]
    L.xjg_worker_stop.restype = None
    L.xjg_worker_stop.argtypes = [vp]
    L.xjg_worker_free.restype = None
    L.xjg_worker_free.argtypes = [vp]
    return L


class Worker:
    """xjg_worker (XJGlue.h:27-32): holds layers [l0, l1) and serves them over the reference's TCP protocol
    (core/xj_net.c:119-292) on a background thread; the stage backend is the build's (CPU or CUDA)."""

    def __init__(self, which: str, path, l0: int, l1: int, port: int, pin: int):
        import threading
        self.L = lib(which)
        err = ctypes.create_string_buffer(512)
        self.w = self.L.xjg_worker_new(str(path).encode(), l0, l1, pin, None, None, err, 512)
        if not self.w:
            raise RuntimeError(err.value.decode(errors="replace"))
        self.port, self.rc, self.err = port, None, ctypes.create_string_buffer(512)
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        self.rc = self.L.xjg_worker_run(self.w, self.port, self.err, 512)

    def close(self):
        if self.w:
            self.L.xjg_worker_stop(self.w)
            self.t.join(timeout=30)
            self.L.xjg_worker_free(self.w)
            self.w = None


class Host:
    """One xjg_host: the whole model on this machine, or layers [s1, s2) on a worker at worker:port."""

    def __init__(self, which: str, path, n_ctx: int = 512, mtp_path=None, draft: int = 0, worker: str = "",
                 port: int = 0, pin: int = 0, s1: int = 0, s2: int = 0):
        self.L = lib(which)
        info, err = ctypes.create_string_buffer(1024), ctypes.create_string_buffer(512)
        self.h = self.L.xjg_host_new(str(path).encode(), worker.encode(), port, pin, s1, s2, n_ctx,
                                     str(mtp_path).encode() if mtp_path else None, draft, info, 1024, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode(errors="replace"))
        self.info = info.value.decode(errors="replace")

    def chat(self, text: str, temperature: float = 0.0, max_tokens: int = 32):
        """One turn; returns (the streamed answer bytes, stats)."""
        pieces = []

        def cb(ctx, s, n):
            pieces.append(ctypes.string_at(s, n))
            return 0

        fn = PIECE(cb)
        st = Stats()
        err = ctypes.create_string_buffer(512)
        if self.L.xjg_host_chat(self.h, text.encode(), temperature, max_tokens, fn, None, ctypes.byref(st), err, 512):
            raise RuntimeError(err.value.decode(errors="replace"))
        return b"".join(pieces), st

    def reset(self):
        err = ctypes.create_string_buffer(512)
        if self.L.xjg_host_reset(self.h, err, 512):
            raise RuntimeError(err.value.decode(errors="replace"))

    def close(self):
        if self.h:
            self.L.xjg_host_free(self.h)
            self.h = None
