"""Build recipe for the C oracle (TEST INFRASTRUCTURE ONLY).

Compiles ``pkv_oracle.c`` into ``oracle/libpkv_oracle.so`` with gcc and
``-ffp-contract=off`` so that no multiply-add is fused.  The reference
itself is Python + NumPy, so there is no ``oracle/_ref`` binary to build:
the reference's algorithm is pinned through golden vectors instead
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "pkv_oracle.c"
LIB = HERE / "libpkv_oracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
           "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
