"""Build recipe of libtmoe.so: every CUDA source under csrc/ compiled for sm_100a with nvcc into
one in-tree shared library (it travels with the repository; no JIT cache)."""
from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtmoe.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(HERE, "..", "include")]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(HERE, "..", "include", "*.h")) + [__file__]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose else []
    objs = [os.path.join(objdir, os.path.basename(src) + ".o") for src in sources()]

    def compile_one(src_obj):
        src, obj = src_obj
        subprocess.run([NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj], check=True)

    # one nvcc per source, as many at once as there are host cores
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        list(pool.map(compile_one, zip(sources(), objs)))
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static", "-lnccl"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
