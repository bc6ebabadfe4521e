"""Builds the native library libcvmm_sm100.so in-tree with nvcc for sm_100a.

The library exports the C ABI declared in include/cvmm_sm100.h. It is built in
place (next to this file) so that it travels with the source tree; nothing is
installed into site-packages.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcvmm_sm100.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
]


def sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh", ".h"))] + [os.path.join(ROOT, "include", "cvmm_sm100.h")]


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force=False, verbose=False, extra=()):
    """Compile libcvmm_sm100.so unless it is newer than every source."""
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, *extra, "-I", os.path.join(ROOT, "include"),
           os.path.join(CSRC, "cvmm_sm100.cu"), "-o", LIB + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    extra = sys.argv[1:]
    build(force=True, verbose=True, extra=extra)
    print("built", LIB)
