"""Shared pytest setup.

* puts the package directory (``pagedkv_fusion``) and the repository root
  (``oracle``) on ``sys.path``;
* registers the ``gpu`` marker: tests that need a CUDA device and the built
  ``libpagedkv_sm100.so``;
* ``rng`` fixture as in the reference's tests/conftest.py:18-20.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "pagedkv-fusion-custom-cuda-kernels-for-kv-cache-eviction-quantized-paged-attention_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built native library")


@pytest.fixture
def rng() -> np.random.Generator:
    return np.random.default_rng(seed=1234)


def sha(*arrays) -> str:
    """Digest of arrays, as written by tests/golden/make_golden.py."""
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def load_golden(name: str):
    return np.load(GOLDEN / f"golden_{name}.npz")


def native_lib_path() -> Path:
    return PKG / "pagedkv_fusion" / "lib" / "libpagedkv_sm100.so"


def ensure_native_built() -> Path:
    """Builds the library if absent (nvcc cross-compiles without a GPU)."""
    lib = native_lib_path()
    if not lib.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("pkv_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return lib


@pytest.fixture(scope="session")
def cuda():
    """The native module on a CUDA device; fails (does not skip) otherwise,
    so a GPU run can never pass on a missing or silently replaced kernel."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    ensure_native_built()
    from pagedkv_fusion import _C
    return _C
