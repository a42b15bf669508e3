"""Build libodyssey_mp.so in-tree with nvcc for sm_100a.

    python -m odyssey_b200.build        (or odyssey_b200.build.build())

Numerics flags: no fast-math, IEEE division and square root, no FMA
contraction (-fmad=false) and no flush-to-zero, so the kernels round every
float32 operation the way the reference's separate tensor ops do.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libodyssey_mp.so")
SOURCES = ["ody_kernels.cu", "ody_capi.cu", "ody_noalloc.cu"]
HEADERS = ["ody_internal.h", "ody_numerics.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=false",
    "-I", os.path.join(ROOT, "include"),
]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [
        os.path.join(ROOT, "include", "odyssey_mp.h"), os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    if not force and not _stale():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc()] + NVFLAGS + ["-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
