"""Build libneedle3.so: the sm_100a CUDA engine plus its C ABI.

Kernels are compiled for sm_100a only, with -fmad=false (a product and an add
stay two roundings unless the source writes __fmaf_rn) and IEEE division and
square root; host code with -ffp-contract=off for the same reason.
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(HERE, "needle_b200")
LIB = os.path.join(OUT_DIR, "libneedle3.so")
BUILD = os.path.join(HERE, "_build")

CU = ["kernels.cu", "tc_prefill.cu", "engine.cu", "ops.cu", "noalloc.cu"]
CPP = ["cact.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build(force: bool = False, verbose: bool = False) -> str:
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)
    ]
    if not force and not _stale(LIB, deps):
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    common = ["-O3", "-std=c++17", "-I", CSRC, "-I", INCLUDE]
    for f in CPP:
        o = os.path.join(BUILD, f + ".o")
        cmd = ["g++", *common, "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-pthread", "-c",
               os.path.join(CSRC, f), "-o", o]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.check_call(cmd)
        objs.append(o)
    for f in CU:
        o = os.path.join(BUILD, f + ".o")
        cmd = [nvcc, *ARCH, *common, "-lineinfo", "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
               "-Xcompiler", "-fPIC,-ffp-contract=off", "-c", os.path.join(CSRC, f), "-o", o]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.check_call(cmd)
        objs.append(o)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lpthread"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
