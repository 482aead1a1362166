"""Builds libspanqr.so (the CUDA kernels and the C ABI of include/spanqr.h) in-tree for sm_100a with nvcc.

    python -m spanqr_b200.build            # incremental
    python -m spanqr_b200.build --force    # rebuild everything

Each .cu under csrc/ is compiled to an object in csrc/_build/, then linked into spanqr_b200/libspanqr.so.
"""
import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = CSRC / "_build"
LIB = PKG / "libspanqr.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime():
    return max(p.stat().st_mtime for p in list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
               + [PKG.parent / "include" / "spanqr.h"])


def build(force=False, verbose=False, ptxas_info=False):
    BUILD.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    hdr = _deps_mtime()
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            continue
        cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "shared"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose, ptxas_info=a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
