"""The reference package, installed unchanged, for the drop-in tests.

``install()`` is the reference's own install (pip, no index, from the
wheelhouse) into ``baseline/_ref`` -- git-ignored, but it travels with the
repository snapshot to a GPU host -- plus the two parts of the reference
tree that pip does not install and the drop-in tests run unchanged: its
``tests/`` directory (the kernel gate ``tests/test_kernels_gpu.py``) and its
vLLM adapter ``integration/vllm/pagedkv_fusion_backend.py``.  Without a GPU
the reference's setup.py installs its pure-Python package only (no ``_C``),
which is what the drop-in test needs: this build's ``_C`` takes the missing
module's place.  ``--no-deps`` because pip cannot resolve the declared
``numpy`` requirement without an index (numpy is present).

``locate()`` returns the installed tree or None; the tests skip without it.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
REF_DIR = ROOT / "baseline" / "_ref"
REF_SOURCE = Path("/root/reference")  # read by install() only
_NEEDED = ("pagedkv_fusion/ops.py", "pagedkv_fusion/reference.py", "pagedkv_fusion/quantize.py",
           "pagedkv_fusion/testing_utils.py", "tests/test_kernels_gpu.py", "tests/conftest.py",
           "integration/vllm/pagedkv_fusion_backend.py")


def locate() -> Path | None:
    if all((REF_DIR / p).is_file() for p in _NEEDED) and not any(
            (REF_DIR / "pagedkv_fusion").glob("_C*.so")):
        return REF_DIR
    return None


def install(quiet: bool = True) -> Path | None:
    """Installs the reference into baseline/_ref when its source tree is
    present and the install is missing; returns the tree or None."""
    if locate() is not None:
        return REF_DIR
    if not (REF_SOURCE / "pagedkv_fusion" / "ops.py").is_file():
        return None
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "src"  # the source tree is read-only; setuptools writes build/
        shutil.copytree(REF_SOURCE, src, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--no-deps", "--find-links", "/opt/wheelhouse", "--target", str(REF_DIR),
               "--upgrade", str(src)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            if not quiet:
                print(r.stdout[-2000:], r.stderr[-2000:])
            return None
        for sub in ("tests", "integration"):
            dst = REF_DIR / sub
            if dst.exists():
                shutil.rmtree(dst)
            shutil.copytree(src / sub, dst, ignore=shutil.ignore_patterns("__pycache__"))
    return locate()


if __name__ == "__main__":
    where = install(quiet=False)
    print(where if where else "reference not installed")
    sys.exit(0 if where else 1)
