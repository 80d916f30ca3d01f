"""Build ``libsparsevox.so`` (the sm_100a CUDA library) in-tree with nvcc.

    python -m mlx_diffuser_b200.csrc.build [--force] [--verbose]

The shared library lands next to the package (``mlx_diffuser_b200/libsparsevox.so``) so it
travels with the source tree; the CUDA runtime is linked statically. ``--verbose`` prints
ptxas register / shared-memory usage per kernel.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libsparsevox.so")
SOURCES = ["api.cu", "kmap.cu", "pool.cu", "topology.cu", "norm.cu", "backward.cu", "wgrad_tc.cu", "halo.cu", "conv_simt.cu", "conv_tc.cu", "conv_dd.cu", "conv_tf32.cu"]
HEADERS = ["common.cuh", "conv.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs() -> list[str]:
    return [os.path.join(HERE, f) for f in SOURCES + HEADERS] + [
        os.path.join(ROOT, "include", "sparsevox.h")
    ]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    obj_dir = os.path.join(HERE, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    common = ARCH + [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-I" + os.path.join(ROOT, "include"),
    ]
    if verbose:
        common.append("-Xptxas=-v")
    objs = [os.path.join(obj_dir, src.replace(".cu", ".o")) for src in SOURCES]

    def compile_one(src_obj):
        src, obj = src_obj
        subprocess.run([nvcc(), *common, "-c", os.path.join(HERE, src), "-o", obj], check=True)

    # one nvcc per translation unit, in parallel (each is single-threaded)
    workers = max(1, min(len(SOURCES), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        list(pool.map(compile_one, zip(SOURCES, objs)))
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
