"""Build libgsq_b200.so (the C-ABI CUDA library) for sm_100a, in-tree.

Usage: python build.py [--force] [-j N]

Steps: generate csrc/_gen/gsq_grids.h from gguf-py, compile every csrc/*.cu
with nvcc (-gencode arch=compute_100a,code=sm_100a -lineinfo -O3) into
_build/*.o, link gsq_b200/_lib/libgsq_b200.so.  Objects are rebuilt when a
source or header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "gsq_b200", "_lib")
LIB = os.path.join(LIB_DIR, "libgsq_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + CSRC, "-I" + INCLUDE]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(CSRC, "_gen", "*.h")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < newest:
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None) -> str:
    sys.path.insert(0, CSRC)
    import gen_tables  # noqa: E402
    gen_tables.main(os.path.join(CSRC, "_gen"))
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra or []), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--xptxas-v", action="store_true", help="print register/spill usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.xptxas_v else []
    print(build(force=args.force or args.xptxas_v, jobs=args.j, extra=extra))
