"""Compile the CUDA library libkmc.so in-tree (sm_100a) from csrc/*.cu.

    python -m mlx_kmeans_b200.build          # or: python mlx_kmeans_b200/build.py

nvcc cross-compiles without a GPU, so this runs on any machine with the CUDA 12.9 toolkit.  Objects are
compiled in parallel and relinked only when a source or header is newer than the library.
"""
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkmc.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libkmc.so")
    return exe


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return (sorted(glob.glob(os.path.join(CSRC, "*.cu*"))) + sorted(glob.glob(os.path.join(CSRC, "*.h")))
            + [os.path.join(ROOT, "include", "kmc.h")])


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(verbose=False, force=False, extra=()):
    """Compile every csrc/*.cu for sm_100a and link libkmc.so (static cudart). Returns the library path."""
    if not force and not extra and up_to_date():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    exe = nvcc()
    srcs = _sources()

    def compile_one(src):
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        cmd = [exe] + ARCH + FLAGS + list(extra) + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(compile_one, srcs))
    tmp = LIB + ".tmp"
    cmd = [exe] + ARCH + ["-shared", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link of libkmc.so failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
