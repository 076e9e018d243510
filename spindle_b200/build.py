"""Builds the spindle-b200 CUDA library for sm_100a into spindle_b200/libspindle_b200.so.

nvcc compiles every csrc/*.cu with relocatable device code and links them into
one shared library exporting the C ABI of include/spindle_gpu.h.  Runs on a
machine without a GPU (nvcc cross-compiles); the .so is built in-tree.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libspindle_b200.so")
OBJ = os.path.join(ROOT, "_build", "obj")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, jobs=8):
    os.makedirs(OBJ, exist_ok=True)
    hdrs = headers() + [os.path.abspath(__file__)]
    objs, procs = [], []
    for src in sources():
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            procs.append((src, subprocess.Popen(cmd)))
            if len(procs) >= jobs:
                s, p = procs.pop(0)
                if p.wait():
                    raise RuntimeError("nvcc failed on " + s)
    for s, p in procs:
        if p.wait():
            raise RuntimeError("nvcc failed on " + s)
    if force or _newer(LIB, objs):
        tmp = LIB + ".tmp.%d" % os.getpid()
        subprocess.run([NVCC, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", tmp, *objs], check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
