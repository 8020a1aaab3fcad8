"""Build the sm_100a shared library ``libexl3_b200.so`` in-tree with nvcc.

The library exports the C ABI declared in ``include/exl3_b200.h``; it is
loaded with ctypes by :mod:`exl3_b200._native`.  The CUDA runtime is linked
statically so the library does not depend on which libcudart the host
process loaded first.
"""

from __future__ import annotations

import os
import shutil
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(ROOT, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libexl3_b200.so")

SOURCES = ["capi.cu", "moe.cu", "reconstruct.cu", "noalloc.cu", "tc_gemm.cu", "ep.cu", "ngram.cu"]
HEADERS = ["exl3_common.cuh", "exl3_internal.h", "tc_common.cuh", "tc_gemm.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the EXL3 CUDA library cannot be built")
    return cand


def _inputs() -> list[str]:
    hdr = os.path.join(os.path.dirname(ROOT), "include", "exl3_b200.h")
    return [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [hdr]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in _inputs() if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
