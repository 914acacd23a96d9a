"""Build the reference r2splat CUDA extension for sm_100a into ``oracle/_ref``.

Test infrastructure only: the built module is the live reference that GPU
parity tests and ``bench.py --impl reference`` compare against.  It is never
part of the product path.

The recipe compiles the reference's own sources where they lie (all
``r2splat/cuda/csrc/*.cpp`` and ``*.cu`` plus ``r2splat/cuda/include``) with
the reference's nvcc flags (``setup.py:23-48``: ``-O3 --use_fast_math
--expt-relaxed-constexpr``) and an explicit ``-gencode`` for sm_100a, through
``torch.utils.cpp_extension.load`` (not the reference's setup.py).  Objects go
to ``oracle/_ref/build``; the module is copied to
``oracle/_ref/r2splat_ref_csrc.so`` so it can travel without the sources.

Usage: ``python oracle/build_ref.py [reference_root]`` (default: the
``BT3DGS_REFERENCE_ROOT`` environment variable, else ``oracle.REFERENCE_ROOT``).
Takes ~6 minutes with 8 cores.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import REFERENCE_ROOT  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE_NAME = "r2splat_ref_csrc"
SO_PATH = os.path.join(OUT_DIR, MODULE_NAME + ".so")


def build(reference_root: str = REFERENCE_ROOT) -> str:
    from torch.utils.cpp_extension import load

    csrc = os.path.join(reference_root, "r2splat", "cuda", "csrc")
    include = os.path.join(reference_root, "r2splat", "cuda", "include")
    if not os.path.isdir(csrc):
        raise FileNotFoundError(f"reference sources not found under {csrc}")
    sources = sorted(glob.glob(os.path.join(csrc, "*.cpp")) + glob.glob(os.path.join(csrc, "*.cu")))
    build_dir = os.path.join(OUT_DIR, "build")
    os.makedirs(build_dir, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    load(
        name=MODULE_NAME,
        sources=sources,
        extra_include_paths=[include],
        extra_cflags=["-O3"],
        extra_cuda_cflags=[
            "-O3",
            "--use_fast_math",
            "--expt-relaxed-constexpr",
            "-gencode=arch=compute_100a,code=sm_100a",
        ],
        build_directory=build_dir,
        verbose=True,
    )
    shutil.copy2(os.path.join(build_dir, MODULE_NAME + ".so"), SO_PATH)
    return SO_PATH


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else REFERENCE_ROOT
    print(build(root))
