"""Build libpagedkv_sm100.so (sm_100a) in-tree.

    python build.py            # incremental
    python build.py --force    # rebuild every object

Each csrc/*.cu is compiled with nvcc for sm_100a (-gencode
arch=compute_100a,code=sm_100a, -O3, -lineinfo, no fast-math: the numerics
contract needs IEEE division and round-half-even), the objects are linked
with a static CUDA runtime, and the library is written to
pagedkv_fusion/lib/libpagedkv_sm100.so, where pagedkv_fusion._C loads it.
The library needs no CUDA driver at load time (driver entry points are
resolved lazily), so it loads on GPU-less build machines too.

csrc/pkv_pycall.c (direct CPython calls into the C ABI for the eviction
latency path) is compiled with the host C compiler against this
interpreter's headers into pagedkv_fusion/lib/_pkv_pycall<ext suffix>,
linked to the library beside it.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB_DIR = HERE / "pagedkv_fusion" / "lib"
LIB = LIB_DIR / "libpagedkv_sm100.so"
INCLUDE = HERE.parent / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I", str(CSRC), "-I", str(INCLUDE)]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed on {src.name}")
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        _build_pycall()
        return LIB
    tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    _build_pycall(force=True)
    return LIB


def pycall_path() -> Path:
    import sysconfig
    return LIB_DIR / ("_pkv_pycall" + sysconfig.get_config_var("EXT_SUFFIX"))


def _build_pycall(force: bool = False) -> Path:
    import sysconfig
    src = CSRC / "pkv_pycall.c"
    out = pycall_path()
    deps = [src, LIB, INCLUDE / "pagedkv_fusion.h"]
    if not force and out.exists() and out.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return out
    tmp = out.with_suffix(f".{os.getpid()}.tmp")
    cmd = [os.environ.get("CC", "gcc"), "-O2", "-shared", "-fPIC", "-std=c11",
           "-I", sysconfig.get_paths()["include"], "-I", str(INCLUDE), str(src), "-o", str(tmp),
           "-L", str(LIB_DIR), "-lpagedkv_sm100", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("compiling pkv_pycall.c failed")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
