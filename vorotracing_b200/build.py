"""Build libvorotracing_b200.so in-tree with nvcc for sm_100a.

    python -m vorotracing_b200.build [--force] [--verbose]

Every .cu under csrc/ is compiled separately (in parallel) into _build/ and
linked into vorotracing_b200/libvorotracing_b200.so.  The traversal files are
built with -fmad=false and without fast math: each binary32 operation is a
separate IEEE round-to-nearest operation, which is what makes the kernels
agree bit for bit with the CPU restatement used by the tests.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libvorotracing_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]


def _deps():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) +
            [os.path.join(ROOT, "include", "vorotracing_b200.h"), __file__])


def _compile(src: str, force: bool, verbose: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(p) for p in [src] + _deps())
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < newest:
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose, list(extra)), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(map(os.path.getmtime, objs)):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register / spill usage")
    args = ap.parse_args()
    print(build(args.force or args.ptxas, args.verbose, ["-Xptxas", "-v"] if args.ptxas else []))
