"""Build libr2s.so, the sm_100a C-ABI library behind the r2splat package.

Every CUDA source under ``csrc/`` is compiled with nvcc for sm_100a
(``-gencode arch=compute_100a,code=sm_100a``) with the arithmetic flags of
the reference build (``-O3 --use_fast_math``: the integer binning outputs
depend on the same float rounding) -- except ``*_precise.cu``, compiled
without fast math to reproduce torch's float kernels -- then linked into
``r2splat/_lib/libr2s.so``.  Objects are cached in ``_build/`` and rebuilt
when a source or header is newer.

``--debug`` builds the bounds-checked library instead: every source with
``-DR2S_DEBUG`` (csrc/r2s_debug.cuh) into ``r2splat/_lib/libr2s_debug.so``
(objects in ``_build_debug/``); load it with ``R2S_LIBRARY=<path>``.

Usage: ``python bt-3dgs_b200/build.py [-j JOBS] [--force] [--debug]``
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
BUILD_DIR = os.path.join(PKG_ROOT, "_build")
LIB_DIR = os.path.join(PKG_ROOT, "r2splat", "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libr2s.so")
DEBUG_BUILD_DIR = os.path.join(PKG_ROOT, "_build_debug")
DEBUG_LIB_PATH = os.path.join(LIB_DIR, "libr2s_debug.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "--use_fast_math",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
] + ARCH


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or add CUDA to PATH")
    return cand


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + _headers())


def build(jobs: int | None = None, force: bool = False, verbose: bool = False,
          debug: bool = False) -> str:
    nvcc = _nvcc()
    build_dir = DEBUG_BUILD_DIR if debug else BUILD_DIR
    lib_path = DEBUG_LIB_PATH if debug else LIB_PATH
    extra = ["-DR2S_DEBUG"] if debug else []
    os.makedirs(build_dir, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(build_dir, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(src, obj):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        flags = NVCC_FLAGS
        if src.endswith("_precise.cu"):
            # accurate libm and IEEE division/sqrt, no flush-to-zero: these
            # kernels reproduce torch's float arithmetic bit for bit
            flags = [f for f in NVCC_FLAGS if f != "--use_fast_math"]
        cmd = [nvcc, *flags, *extra, "-I", INCLUDE, "-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [nvcc, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
                   "-fvisibility=hidden", *extra, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
        return res.stderr

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
            for out in ex.map(compile_one, todo):
                if out and verbose:
                    print(out, file=sys.stderr)
    if todo or not os.path.exists(lib_path):
        tmp = lib_path + ".tmp"
        cmd = [nvcc, "-shared", *ARCH, "-o", tmp, *objs, "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--debug", action="store_true", help="bounds-checked build (R2S_DEBUG)")
    a = ap.parse_args()
    print(build(a.jobs, a.force, a.verbose, a.debug))
