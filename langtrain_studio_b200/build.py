"""Build the native library (liblt_kv.so) in-tree with nvcc for sm_100a.

The library is the product: C++ host bookkeeping + sm_100a CUDA kernels
behind the C ABI declared in include/lt_kv.h.  It is built into
langtrain_studio_b200/lib/ so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "liblt_kv.so"

SOURCES = [CSRC / "lt_kv_kernels.cu", CSRC / "lt_kv.cpp", CSRC / "lt_kv_nccl.cpp", CSRC / "lt_kv_noalloc.cu",
           CSRC / "lt_llama.cu", CSRC / "lt_sched.cpp"]
HEADERS = [CSRC / "lt_kv_internal.h", INCLUDE / "lt_kv.h", INCLUDE / "lt_llama.h", INCLUDE / "lt_sched.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall", "-shared",
              "--expt-relaxed-constexpr", "-ldl"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblt_kv.so")


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile liblt_kv.so if it is missing or older than its sources."""
    if not force and not stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp%d" % os.getpid())
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-o", str(tmp),
           *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
