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
# Measurement build: the same sources with the reference's compiler flags
# (-use_fast_math, contraction on) and VT_REF_FASTMATH; loaded only by tests
# that bound the gap between exact and fast-math arithmetic.
LIB_REFMATH = os.path.join(HERE, "libvorotracing_b200_refmath.so")
REFMATH_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-use_fast_math", "-fmad=true",
                 "-DVT_REF_FASTMATH", "-Xcompiler", "-fPIC", "-Xcompiler",
                 "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]
REFMATH_SOURCES = ("vt_abi.cu", "vt_pack.cu", "vt_infer.cu", "vt_train.cu")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]


def _deps():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) +
            [os.path.join(ROOT, "include", "vorotracing_b200.h"), __file__])


def _compile(src: str, force: bool, verbose: bool, extra, build_dir=BUILD, flags=FLAGS) -> str:
    obj = os.path.join(build_dir, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(p) for p in [src] + _deps())
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < newest:
        cmd = [NVCC, *ARCH, *flags, *extra, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return obj


def build(force: bool = False, verbose: bool = False, extra=(), refmath: bool = False) -> str:
    """Build the library (refmath=True: the fast-math measurement build)."""
    lib = LIB_REFMATH if refmath else LIB
    build_dir = os.path.join(BUILD, "refmath") if refmath else BUILD
    flags = REFMATH_FLAGS if refmath else FLAGS
    os.makedirs(build_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    if refmath:  # the traversal and training kernels; the rest has no float maths to compare
        srcs = [s for s in srcs if os.path.basename(s) in REFMATH_SOURCES]
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose, list(extra), build_dir, flags),
                           srcs))
    if force or not os.path.exists(lib) or os.path.getmtime(lib) < max(map(os.path.getmtime, objs)):
        tmp = lib + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register / spill usage")
    ap.add_argument("--refmath", action="store_true", help="the fast-math measurement build")
    args = ap.parse_args()
    print(build(args.force or args.ptxas, args.verbose, ["-Xptxas", "-v"] if args.ptxas else [],
                refmath=args.refmath))
