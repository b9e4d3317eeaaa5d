"""Build libmoteopt.so (the CUDA kernels and the C ABI of include/moteopt.h) for sm_100a, in-tree.

    python -m mote_b200.build            # or: python mote_b200/build.py

nvcc cross-compiles without a GPU. The library links the CUDA runtime statically and takes the driver's
cuTensorMapEncodeTiled through cudaGetDriverEntryPoint, so it needs no -lcuda at link time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmoteopt.so"
CHECKED_LIB = PKG / "libmoteopt_checked.so"   # the same library with MOTE_OPT_CHECKS: index checks in every kernel
SOURCES = [CSRC / "moteopt.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "moteopt.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found (set NVCC=...)")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None, checked: bool = False) -> Path:
    """nvcc the library; `checked` builds libmoteopt_checked.so, which counts failed index checks
    (moteopt_check_count) instead of the release library."""
    out = CHECKED_LIB if checked else LIB
    if not force and not checked and not needs_build():
        return LIB
    if checked:
        extra = ["-DMOTE_OPT_CHECKS", *(extra or [])]
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", str(ROOT / "include"), "-I", str(CSRC), "--expt-relaxed-constexpr", "-o", str(tmp),
           *[str(s) for s in SOURCES], *(extra or [])]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(force=True, verbose=v, extra=extra, checked="--checked" in sys.argv))
