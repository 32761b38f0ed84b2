"""Builds libcutile_b200.so in-tree from csrc/*.cu for sm_100a with nvcc.

Usage: python cutile-triton_b200/build.py [--force]
The library is rebuilt when any source or the public header is newer than it.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "cutile_b200", "libcutile_b200.so")
HEADER = os.path.join(ROOT, "include", "cutile_b200.h")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    # IEEE semantics: no flush-to-zero, exact division/sqrt (vadd is bit-exact).
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-I" + os.path.join(ROOT, "include"),
]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _needs(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, defines=(), lib=None, obj=None):
    """Compiles every csrc/*.cu and links the library. `defines` (e.g.
    ["CTB_FMHA_EMU_EVERY=2"]) override compile-time tunables; with them, pass
    a separate `lib`/`obj` so the default build is left untouched."""
    global OBJ, LIB
    OBJ = obj or OBJ
    LIB = lib or LIB
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")] + [HEADER]
    objs = []
    for src in sources():
        o = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(o)
        if force or _needs(o, [src] + headers):
            cmd = [NVCC] + FLAGS + ["-D" + d for d in defines] + ["-c", src, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    if force or _needs(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
