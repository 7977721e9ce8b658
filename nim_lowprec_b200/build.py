"""Build liblowprec_cuda.so in-tree with nvcc for sm_100a.

    python nim_lowprec_b200/build.py [--force] [-v]

(Run it by path: importing the package itself loads the built library.)

Every .cu under csrc/ is compiled for `sm_100a` only (the library uses
tcgen05/TMA-era PTX: bulk copies, mbarrier waits, f32x2 arithmetic) and
linked into one shared object next to this file, with the CUDA runtime linked
statically.  The result travels with the repository snapshot; nothing is
installed into site-packages.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(HERE, "liblowprec_cuda.so")
OBJDIR = os.path.join(HERE, "_build")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: ptxas may otherwise contract a multiply feeding an add into one
# FMA even across the explicit mul.rn/add.rn f32x2 pairs of the bit-exact
# paths (measured on sm_100a); this is the device-side twin of the
# reference's -ffp-contract=off (simd/dequant.nim:36).
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    objs = []
    for src in sources():
        obj = os.path.join(OBJDIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-ldl"]
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
