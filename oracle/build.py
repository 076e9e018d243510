"""Build recipe for the CPU oracle (test infrastructure, not product code).

Compiles oracle/*.c with gcc into oracle/_build/libsg_oracle.so.  The flags
matter for parity: -ffp-contract=off keeps gcc from fusing a*b+c (rustc never
does), and the AVX2/FMA/F16C target attributes live in the sources.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libsg_oracle.so")
SOURCES = ["gen.c", "q8k.c", "floatk.c", "pool.c", "kquant.c", "moe.c", "forward.c", "libm.c", "synth.c"]
CFLAGS = ["-O3", "-std=gnu11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
          "-Wall", "-Wno-unused-function", "-pthread"]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = SOURCES + ["sg_oracle.h", "build.py"]
    return any(os.path.getmtime(os.path.join(HERE, s)) > t for s in deps)


def build(force: bool = False) -> str:
    if not force and not stale():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + ".tmp.%d" % os.getpid()
    cmd = ["gcc", *CFLAGS, "-o", tmp, *[os.path.join(HERE, s) for s in SOURCES], "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
