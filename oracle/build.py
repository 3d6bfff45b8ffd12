"""Build recipe for the C oracle (test infrastructure only).

    python oracle/build.py

compiles oracle/scan_oracle.c with gcc into oracle/_build/libscan_oracle.so.
The reference (Anamaya1729/mamba-metal-scan) is pure Python plus Metal shader
source, so there is no reference C/C++ to compile into oracle/_ref; the
reference itself is exercised only through the golden vectors in tests/golden.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "scan_oracle.c"
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "libscan_oracle.so"


def build(force: bool = False, verbose: bool = False) -> Path:
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    tmp = OUT_DIR / f".libscan_oracle.{os.getpid()}.so"
    cmd = ["gcc", "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared",
           "-fno-fast-math", "-ffp-contract=off",
           str(SRC), "-o", str(tmp), "-lm"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)           # atomic: concurrent builders never see half a file
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
