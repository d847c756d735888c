"""Synthetic qwen35 GGUF models for tests and benchmarks (ctypes front end of synth/libxj_synth.so).

The named configurations are the workloads of the decode benchmark suite:

- ``CONFIG0``: tiny 4-layer hybrid (3 Gated-DeltaNet + 1 gated GQA), E=512, 8 heads x 64 (2 KV heads),
  GDN 4 key heads / 8 value heads x 64, FFN 1408, vocab 8192, every 2-D weight Q8_0.
- ``CONFIG3``: ~2B-class hybrid, 28 layers (21 GDN + 7 GQA), E=2048, 16 q / 4 KV heads x 128,
  GDN 16 x 128, FFN 6144, vocab 151936, Q4_K_M policy (Q6_K embeddings/head, Q6_K ffn_down and
  attn_v on the "more bits" layers).
- ``DRAFT``: the config-0 architecture widened to E=1024 / 8 layers, Q8_0, vocab of CONFIG3.
- ``MID``: CONFIG3's head shapes and Q4_K_M policy at test size: 8 layers (6 GDN + 2 GQA), E=512,
  4 q / 2 KV heads x 128, GDN 4 x 128, FFN 1536, vocab 4096.
"""
from __future__ import annotations

import ctypes
import dataclasses
import hashlib
import os
import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "synth" / "libxj_synth.so"

# ggml type ids (include/xj_abi.h)
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30


class _Config(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int), ("n_embd", ctypes.c_int), ("n_ff", ctypes.c_int), ("n_vocab", ctypes.c_int),
        ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int), ("head_dim", ctypes.c_int), ("n_rot", ctypes.c_int),
        ("rope_base", ctypes.c_float), ("eps", ctypes.c_float),
        ("conv_k", ctypes.c_int), ("s_k", ctypes.c_int), ("h_k", ctypes.c_int), ("h_v", ctypes.c_int),
        ("full_attn_interval", ctypes.c_int),
        ("wtype", ctypes.c_int), ("io_type", ctypes.c_int), ("tied", ctypes.c_int), ("mtp", ctypes.c_int),
        ("fused_qkv", ctypes.c_int),
        ("seed", ctypes.c_ulonglong), ("w_std", ctypes.c_float),
    ]


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layer: int = 4
    n_embd: int = 512
    n_ff: int = 1408
    n_vocab: int = 8192
    n_head: int = 8
    n_head_kv: int = 2
    head_dim: int = 64
    n_rot: int = 16
    rope_base: float = 1e6
    eps: float = 1e-6
    conv_k: int = 4
    s_k: int = 64
    h_k: int = 4
    h_v: int = 8
    full_attn_interval: int = 4
    wtype: int = Q8_0
    io_type: int = -1
    tied: bool = False
    mtp: bool = False
    fused_qkv: bool = False
    seed: int = 20261201
    w_std: float = 0.02

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def _c(self) -> _Config:
        c = _Config()
        for f in _Config._fields_:
            k = f[0]
            v = getattr(self, k)
            setattr(c, k, int(v) if isinstance(v, bool) else v)
        return c


CONFIG0 = ModelConfig("config0-tiny-q8_0")
CONFIG3 = ModelConfig(
    "config3-2b-q4_k_m", n_layer=28, n_embd=2048, n_ff=6144, n_vocab=151936, n_head=16, n_head_kv=4,
    head_dim=128, n_rot=32, s_k=128, h_k=16, h_v=16, wtype=Q4_K)
MID = ModelConfig("mid-q4_k_m", n_layer=8, n_embd=512, n_ff=1536, n_vocab=4096, n_head=4, n_head_kv=2,
                  head_dim=128, n_rot=32, s_k=128, h_k=4, h_v=4, wtype=Q4_K)
# a small draft for MID (same vocabulary), for the speculative-decoding tests
MID_DRAFT = ModelConfig("mid-draft-q8_0", n_layer=4, n_embd=256, n_ff=512, n_vocab=4096, n_head=2, n_head_kv=1,
                        head_dim=128, n_rot=32, s_k=64, h_k=2, h_v=4, wtype=Q8_0, seed=20261202)
DRAFT = ModelConfig("draft-1024-q8_0", n_layer=8, n_embd=1024, n_ff=2816, n_vocab=151936, n_head=8,
                    n_head_kv=2, head_dim=128, n_rot=32, s_k=128, h_k=4, h_v=8, wtype=Q8_0)


def _lib() -> ctypes.CDLL:
    if not LIB.exists():
        subprocess.run(["make", "-C", str(LIB.parent), "CXX=g++"], check=True, capture_output=True)
    lib = ctypes.CDLL(str(LIB))
    lib.xjs_write_gguf.restype = ctypes.c_longlong
    lib.xjs_write_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Config), ctypes.c_int, ctypes.c_char_p,
                                   ctypes.c_int]
    lib.xjs_quantize_row.restype = ctypes.c_int
    lib.xjs_quantize_row.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]
    return lib


def write_gguf(path: str | os.PathLike, cfg: ModelConfig, threads: int = 0) -> int:
    """Write the seeded model `cfg` to `path`; returns the file size in bytes."""
    err = ctypes.create_string_buffer(256)
    c = cfg._c()
    n = _lib().xjs_write_gguf(str(path).encode(), ctypes.byref(c), threads, err, 256)
    if n < 0:
        raise RuntimeError(err.value.decode())
    return n


def model_path(cfg: ModelConfig, directory: str | os.PathLike | None = None) -> pathlib.Path:
    """Where cached_gguf keeps `cfg` (default directory: $XJ_MODEL_DIR or /tmp/xj_models); nothing is written."""
    d = pathlib.Path(directory or os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models"))
    key = hashlib.sha1(repr(dataclasses.astuple(cfg)).encode()).hexdigest()[:12]
    return d / f"{cfg.name}-{key}.gguf"


def cached_gguf(cfg: ModelConfig, directory: str | os.PathLike | None = None) -> pathlib.Path:
    """Path of `cfg` written once into `directory` (default: $XJ_MODEL_DIR or /tmp/xj_models)."""
    p = model_path(cfg, directory)
    p.parent.mkdir(parents=True, exist_ok=True)
    if not p.exists():
        tmp = p.with_suffix(f".tmp{os.getpid()}")
        write_gguf(tmp, cfg)
        os.replace(tmp, p)
    return p


def quantize_row(type_id: int, x) -> bytes:
    """Quantise a 1-D float32 array (length a multiple of the block size) with the writer's quantiser."""
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    blk = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176),
           Q6_K: (256, 210)}[type_id]
    out = np.zeros(x.size // blk[0] * blk[1], dtype=np.uint8)
    if _lib().xjs_quantize_row(type_id, x.ctypes.data, out.ctypes.data, x.size) != 0:
        raise ValueError("row length is not a multiple of the block size")
    return out.tobytes()
