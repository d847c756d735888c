"""Host-side checks of libxj_cuda.so that need no GPU: the library loads and exports every symbol
include/*.h declares, include/xj_abi.h has the runtime's struct layout, and the library's GGUF loader
and embedding lookup agree with the runtime's (core/xj_model.c, core/xj_cpu.c:369-373)."""
from __future__ import annotations

import ctypes
import pathlib
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle import xj_oracle as xo

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = re.sub(r"//[^\n]*", "", h.read_text())
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(xj\w*)\s*\(", text, re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from xjb200 import xjcuda
    lib = xjcuda.lib()
    names = declared_functions()
    assert "xj_cuda_stage_new" in names and "xjc_model_load" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


ABI_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "xj_abi.h"
int main(void) {
    printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n",
        sizeof(xj_w), sizeof(xj_layer), sizeof(xj_hparams), sizeof(xj_model), sizeof(xj_stage),
        offsetof(xj_model, layers), offsetof(xj_model, fingerprint), offsetof(xj_model, mtp_eh),
        offsetof(xj_stage, forward), offsetof(xj_stage, impl), offsetof(xj_stage, keep),
        offsetof(xj_layer, ssm_qkv), offsetof(xj_model, has_mtp), sizeof(gguf_file), offsetof(xj_stage, backend));
    return 0;
}
"""


def test_abi_matches_reference_layout(ref_lib, tmp_path):
    src = tmp_path / "abi.c"
    src.write_text(ABI_PROBE)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), "-o", str(exe), str(src)], check=True)
    mine = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    theirs = [ref_lib.lib().xjr_abi(i) for i in range(15)]
    assert mine == theirs


def _hp(model_ptr):
    from xjb200 import xjcuda
    return xjcuda._Model.from_address(model_ptr).hp


@pytest.mark.parametrize("which", ["tiny", "config0"])
def test_loader_matches_reference(ref_lib, golden, tiny_path, config0_path, which):
    from xjb200 import xjcuda
    path = tiny_path if which == "tiny" else config0_path
    mine = xjcuda.Model(path)
    theirs = ref_lib.Model(path)
    a, b = _hp(mine.ptr), _hp(theirs.ptr)
    for f, _ in xjcuda._HParams._fields_:
        assert getattr(a, f) == getattr(b, f), f
    assert mine.m.fingerprint == theirs.fingerprint == int(golden[f"{which}_fingerprint"])
    assert mine.m.has_mtp == theirs.has_mtp
    assert ctypes.sizeof(xjcuda._Model) == ref_lib.lib().xjr_abi(3)
    assert xjcuda._Model.fingerprint.offset == ref_lib.lib().xjr_abi(6)
    for tok in (0, 1, mine.n_vocab - 1, mine.n_vocab, -1, 123):
        e1, e2 = mine.embed(tok), theirs.embed(tok)
        assert e1.view(np.uint32).tolist() == e2.view(np.uint32).tolist(), tok


def test_loader_embed_matches_oracle_without_reference(golden, config0_path):
    from xjb200 import xjcuda
    mine = xjcuda.Model(config0_path)
    om = xo.Model(config0_path)
    for tok in (0, 5, 8191, 8192):
        assert mine.embed(tok).view(np.uint32).tolist() == om.embed(tok).view(np.uint32).tolist()
    assert mine.m.fingerprint == int(golden["config0_fingerprint"])


def test_loader_errors(tmp_path, tiny_path):
    from xjb200 import xjcuda
    with pytest.raises(xjcuda.XjError):
        xjcuda.Model(tmp_path / "missing.gguf")
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(100))
    with pytest.raises(xjcuda.XjError, match="GGUF"):
        xjcuda.Model(bad)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(pathlib.Path(tiny_path).read_bytes()[:5000])
    with pytest.raises(xjcuda.XjError):
        xjcuda.Model(cut)


def test_reference_session_layer_runs_on_cpu(tiny_path):
    """The session-layer build the GPU test compares against (XJGlue.c with CPU stages) chats here."""
    from oracle import glue
    if not glue.available("cpu"):
        pytest.skip("session-layer build missing")
    h = glue.Host("cpu", tiny_path, 256)
    try:
        ans, st = h.chat("hello", 0.0, 8)
        assert st.prompt_tokens > 0 and st.gen_tokens >= 0 and st.n_past >= st.prompt_tokens
    finally:
        h.close()
