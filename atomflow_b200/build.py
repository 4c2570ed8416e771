"""Build the CUDA library in-tree for sm_100a.

    python -m atomflow_b200.build          # -> atomflow_b200/libatomflow_b200.so

nvcc cross-compiles without a GPU, so this runs on any machine with CUDA 12.8+.
The shared CUDA runtime is linked so the library shares the process's current
device and streams with any other CUDA user in the process (e.g. PyTorch).
"""
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libatomflow_b200.so"
CLI = PKG / "af_generate"        # the C++ greedy-decode driver on the C ABI
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-cudart", "shared"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return (sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp")) +
            sorted((ROOT / "include").glob("*.h")))


def up_to_date() -> bool:
    if not LIB.exists() or not CLI.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers())


# Translation units whose element-wise arithmetic must round exactly like the
# reference's kernels, which are built with --use_fast_math (flush-to-zero and
# the approximate exp / reciprocal / rsqrt forms): the decode-step kernels.
FAST_MATH = {"af_decode.cu"}


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIB.with_suffix(".so.tmp")
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        extra = ["--use_fast_math"] if src.name in FAST_MATH else []
        cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", "-I", str(ROOT / "include"), "-o", str(obj), str(src)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True, cwd=str(PKG))
        objs.append(str(obj))
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=str(PKG))
    os.replace(tmp, LIB)
    cmd = [nvcc, *ARCH, "-O2", "-std=c++17", "-I", str(ROOT / "include"), "-o", str(CLI),
           str(CSRC / "af_generate.cpp"), "-L", str(PKG), "-latomflow_b200", "-cudart", "shared",
           "-Xlinker", "-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=str(PKG))
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
