"""Builds the in-tree CUDA library `lib/libsinkcache_b200.so` with nvcc for sm_100a.

    python -m attention_sinks_b200.build [--force]

The library exports the C ABI declared in include/sinkcache_b200.h.  It links the CUDA
runtime statically, so it needs nothing at run time beyond the driver.
"""

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
SOURCES = [os.path.join(CSRC, "sinkcache_b200.cu")]
# every header the translation unit includes: a change to any of them rebuilds the library
HEADERS = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))
LIB = os.path.join(HERE, "lib", "libsinkcache_b200.so")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a CUDA library cannot be built")


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    built = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= built for p in SOURCES + HEADERS + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library unless it is newer than every source; returns its path."""
    if not force and up_to_date():
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *SOURCES, "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
