"""Build libmms_scan.so (the sm_100a selective-scan library) in-tree.

    python mamba-metal-scan_b200/build.py [--force] [--verbose]

nvcc compiles csrc/*.cu for sm_100a only and links them into
mamba_metal/lib/libmms_scan.so, next to the Python package that loads it.
The library is plain C ABI (include/mms_scan.h); it links the CUDA runtime
statically so it loads without a matching libcudart on the library path.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PKG_ROOT / "mamba_metal" / "lib"
LIB = LIB_DIR / "libmms_scan.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in
                 list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)])
    return LIB.stat().st_mtime < newest


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_DIR / f".libmms_scan.{os.getpid()}.so"
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           "-I", str(INCLUDE), "-I", str(CSRC)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in sources()] + ["-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
