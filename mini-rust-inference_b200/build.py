"""Builds libmri_gpu.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python mini-rust-inference_b200/build.py [--force]

Each csrc/*.cu compiles to an object under _build/ (parallel, incremental on
source/header mtimes), then links into mini-rust-inference_b200/libmri_gpu.so.
-fmad=false keeps every float multiply-add that is not an explicit
__fmaf_rn as two IEEE roundings, as in the reference's Rust arithmetic.
"""
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmri_gpu.so")
INCLUDE = os.path.join(REPO, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-cudart", "static", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(INCLUDE, "mri_gpu.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [NVCC] + ARCH + FLAGS + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if "-Xptxas" in os.environ.get("MRI_NVCC_EXTRA", ""):
            sys.stdout.write(r.stdout + r.stderr)
    return obj


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(_compile, srcs))
    if force or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
