"""Build the native library (liblt_kv.so) in-tree with nvcc for sm_100a.

The library is the product: C++ host bookkeeping + sm_100a CUDA kernels
behind the C ABI declared in include/lt_kv.h.  It is built into
langtrain_studio_b200/lib/ so it travels with the source tree.

Two debug variants of the same sources sit beside it:
  checked  liblt_kv_checked.so  -DLT_BOUNDS_CHECK: the kernels test every
           block id they read from a device table against the pool and
           report a bad one (LT_E_BOUNDS) instead of reading outside it;
  asan     liblt_kv_asan.so     host code under AddressSanitizer and
           UndefinedBehaviorSanitizer (the C++ bookkeeping, scheduler and
           ABI glue); load it into a process started with libasan preloaded.
The environment variable LT_KV_VARIANT (release | checked | asan) picks the
one langtrain_studio_b200._native loads.
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
VARIANTS = {
    "release": (LIB, []),
    "checked": (LIB_DIR / "liblt_kv_checked.so", ["-DLT_BOUNDS_CHECK"]),
    "asan": (LIB_DIR / "liblt_kv_asan.so",
             ["-Xcompiler", "-fsanitize=address,-fsanitize=undefined,-fno-omit-frame-pointer,-fno-sanitize-recover=all",
              "-lasan", "-lubsan"]),
}

SOURCES = [CSRC / "lt_kv_kernels.cu", CSRC / "lt_kv.cpp", CSRC / "lt_kv_nccl.cpp", CSRC / "lt_kv_noalloc.cu",
           CSRC / "lt_llama.cu", CSRC / "lt_llama_decode.cu", CSRC / "lt_sched.cpp", CSRC / "lt_prefix.cpp"]
HEADERS = [CSRC / "lt_kv_internal.h", CSRC / "lt_kv_layout.cuh", CSRC / "lt_q8_device.cuh", CSRC / "lt_llama_decode.h",
           INCLUDE / "lt_kv.h", INCLUDE / "lt_llama.h", INCLUDE / "lt_sched.h", INCLUDE / "lt_prefix.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall", "-shared",
              "--expt-relaxed-constexpr", "-ldl"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblt_kv.so")


def library(variant: str = "release") -> Path:
    if variant not in VARIANTS:
        raise ValueError(f"unknown library variant {variant!r} (one of {sorted(VARIANTS)})")
    return VARIANTS[variant][0]


def stale(variant: str = "release") -> bool:
    lib = library(variant)
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS + [Path(__file__)])


def build(force: bool = False, verbose: bool = False, variant: str = "release") -> Path:
    """Compile the library variant if it is missing or older than its sources."""
    lib = library(variant)
    if not force and not stale(variant):
        return lib
    LIB_DIR.mkdir(exist_ok=True)
    tmp = lib.with_suffix(".so.tmp%d" % os.getpid())
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *VARIANTS[variant][1], "-I", str(INCLUDE), "-I", str(CSRC), "-o", str(tmp),
           *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    import sys

    for v in sys.argv[1:] or ["release"]:
        print(build(force=True, verbose=True, variant=v))
