"""Build libmoteopt.so (the CUDA kernels and the C ABI of include/moteopt.h) for sm_100a, in-tree.

    python -m mote_b200.build            # or: python mote_b200/build.py
    python -m mote_b200.build --checked  # libmoteopt_checked.so

The release build keeps ptxas's per-kernel resource report (registers, spills, shared memory) in
mote_b200/_build/ptxas_release.txt.

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
RESOURCES = PKG / "_build" / "ptxas_release.txt"   # ptxas's per-kernel registers / spills of the release build
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
    else:   # keep ptxas's resource report (registers, spills, shared memory per kernel) beside the build
        extra = ["-Xptxas", "-v", *(extra or [])]
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", str(ROOT / "include"), "-I", str(CSRC), "--expt-relaxed-constexpr", "-o", str(tmp),
           *[str(s) for s in SOURCES], *(extra or [])]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise subprocess.CalledProcessError(r.returncode, cmd)
    if not checked:
        RESOURCES.parent.mkdir(exist_ok=True)
        RESOURCES.write_text(r.stderr + r.stdout)
    elif verbose:
        sys.stderr.write(r.stderr)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(force=True, verbose=v, checked="--checked" in sys.argv))
