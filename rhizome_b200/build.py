"""Builds librhizome_gdr.so in-tree for sm_100a with nvcc.

The library is plain CUDA C++ behind a C ABI (include/rhizome_gdr.h); torch is
not linked. Run `python -m rhizome_b200.build` or call build().
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIB_DIR, "librhizome_gdr.so")
HEADER = os.path.join(ROOT, "include", "rhizome_gdr.h")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the GDR library needs the CUDA 12.9 toolkit to build")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps.append(HEADER)
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu under csrc/ into one shared library (in-tree)."""
    if not force and not _stale():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(PKG, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = _nvcc()
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
        objs.append(obj)
        procs.append((src, subprocess.Popen([nvcc, *flags, "-c", src, "-o", obj])))
    failed = [src for src, p in procs if p.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed on {failed}")
    tmp = LIB + f".tmp{os.getpid()}"
    subprocess.run([nvcc, *ARCH, "-shared", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
