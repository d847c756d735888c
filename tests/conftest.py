"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on a CPU-only machine."""
from __future__ import annotations

import importlib.util
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(GOLDEN))


def load_pkg():
    """Import the package folder meta-work_b200/ under the name `xjb200`."""
    if "xjb200" in sys.modules:
        return sys.modules["xjb200"]
    spec = importlib.util.spec_from_file_location("xjb200", ROOT / "meta-work_b200" / "__init__.py",
                                                  submodule_search_locations=[str(ROOT / "meta-work_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xjb200"] = mod
    spec.loader.exec_module(mod)
    return mod


load_pkg()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def tiny_path():
    return GOLDEN / "tiny_mtp.gguf"


@pytest.fixture(scope="session")
def config0_path(tmp_path_factory):
    from xjb200 import synth
    return synth.cached_gguf(synth.CONFIG0, tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def mid_path(tmp_path_factory):
    from xjb200 import synth
    return synth.cached_gguf(synth.MID, tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def mid_draft_path(tmp_path_factory):
    from xjb200 import synth
    return synth.cached_gguf(synth.MID_DRAFT, tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def ref_lib():
    from oracle import ref
    if not ref.available() and not ref.build():
        pytest.skip("reference library oracle/_ref/libxjref.so not built")
    return ref


def rel_err(a, b) -> float:
    """max|a-b| / max|b| (tools/xjpipe-check.c:17-25)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.abs(a - b).max()
    m = np.abs(b).max()
    return float(d / m if m > 0 else d)
