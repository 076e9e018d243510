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


def sources(csrc=CSRC):
    return sorted(glob.glob(os.path.join(csrc, "*.cu")))


def headers(csrc=CSRC):
    return sorted(glob.glob(os.path.join(csrc, "*.cuh")) + glob.glob(os.path.join(csrc, "*.h")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, jobs=8, csrc=CSRC, lib=LIB, obj_dir=OBJ):
    """Compiles csrc/*.cu into lib (defaults: this package's sources and .so)."""
    os.makedirs(obj_dir, exist_ok=True)
    hdrs = headers(csrc) + [os.path.abspath(__file__)]
    objs, procs = [], []
    for src in sources(csrc):
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
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
    if force or _newer(lib, objs):
        tmp = lib + ".tmp.%d" % os.getpid()
        subprocess.run([NVCC, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", tmp, *objs], check=True)
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--src", default=CSRC, help="directory of .cu sources")
    ap.add_argument("--out", default=LIB, help="shared library to write")
    args = ap.parse_args()
    od = OBJ if args.src == CSRC else os.path.join(os.path.dirname(os.path.abspath(args.out)), "obj")
    print(build(force=args.force, verbose=args.v, csrc=os.path.abspath(args.src), lib=os.path.abspath(args.out),
                obj_dir=od))
