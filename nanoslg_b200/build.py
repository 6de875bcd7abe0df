"""Builds the native library ``nanoslg_b200/lib/libnslg_b200.so`` for sm_100a.

Each ``csrc/*.cu`` file is compiled by nvcc into ``_build/`` (in parallel, skipped
when up to date) and the objects are linked into one shared library that exports the
C ABI of ``include/nslg_b200.h``.  nvcc cross-compiles, so this runs without a GPU.

    python -m nanoslg_b200.build [--force] [--verbose]
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libnslg_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC] + ARCH


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, verbose, extra):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc(), "-c", src, "-o", obj] + NVCC_FLAGS + extra
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)
    return obj


def build(force=False, verbose=False, extra=()):
    """Compiles every csrc/*.cu and links the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose, list(extra)), srcs))
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-Xcompiler", "-fPIC"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/smem per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
