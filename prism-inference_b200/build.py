"""Build libprism_b200.so in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind the C ABI in include/prism_b200.h:
no PyTorch, no JIT cache.  The built .so sits next to this file so it
travels with the repository snapshot to a GPU box.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libprism_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

SOURCES = ["prism_b200.cu", "synth.cu", "static_scratch.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", "--expt-relaxed-constexpr", "-fmad=false"]


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def deps():
    out = []
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".cu", ".cuh", ".h")):
                out.append(os.path.join(d, f))
    return out


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in deps() + [__file__])


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    cmd = [NVCC] + ARCH + FLAGS + ["-I", os.path.join(ROOT, "include"), "-o", LIB] + sources()
    if verbose:
        cmd += ["-Xptxas", "-v"]
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
