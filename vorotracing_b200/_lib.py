"""ctypes binding of libvorotracing_b200.so (the C ABI in include/vorotracing_b200.h).

The shared library is the only compute path: if it is missing or fails to
load, every operator raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvorotracing_b200.so")

_lib = None


class VtScene(C.Structure):
    _fields_ = [("points", C.c_void_p), ("density", C.c_void_p), ("offsets", C.c_void_p),
                ("faces", C.c_void_p), ("num_points", C.c_uint32),
                ("num_face_rows", C.c_uint64)]


class VtPath(C.Structure):
    _fields_ = [("steps", C.c_void_p), ("cap", C.c_uint32), ("len", C.c_void_p)]


class VtDebug(C.Structure):
    _fields_ = [("seq", C.c_void_p), ("seq_cap", C.c_uint32), ("seq_len", C.c_void_p),
                ("stats", C.c_void_p), ("num_intersections", C.c_void_p),
                ("visited", C.c_void_p), ("textured", C.c_void_p)]


PEER_MAX = 8


class VtPeerGrads(C.Structure):
    _fields_ = [("world", C.c_uint32), ("num_points", C.c_uint32), ("res", C.c_int32),
                ("workspace", C.c_void_p * PEER_MAX), ("bucket", C.c_void_p * PEER_MAX),
                ("staging", C.c_void_p * PEER_MAX)]


def load(path: str = LIB_PATH, require_all: bool = True):
    """Open a build of the library and declare the non-int return types.
    require_all: every entry point the header declares must be exported."""
    if not os.path.exists(path):
        raise RuntimeError(
            f"vorotracing_b200: CUDA library not built ({path}); run "
            "`python -m vorotracing_b200.build` (there is no CPU fallback)")
    L = C.CDLL(path)
    L.vt_last_error.restype = C.c_char_p
    L.vt_version.restype = C.c_char_p
    L.vt_face_rows.restype = C.c_uint64
    L.vt_face_rows.argtypes = [C.c_uint64]
    L.vt_adj_diff_rows.restype = C.c_uint64
    L.vt_adj_diff_rows.argtypes = [C.c_uint64]
    if require_all:
        for name in exported_symbols():
            getattr(L, name)  # every declared entry point must be exported
    for name in ("vt_bvh_nodes_bytes", "vt_bvh_workspace_bytes", "vt_morton_workspace_bytes",
                 "vt_trace_bwd_workspace_bytes", "vt_peer_staging_floats"):
        if hasattr(L, name):
            getattr(L, name).restype = C.c_uint64
    return L


def lib():
    """Load the library (raises RuntimeError when it is absent)."""
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


class using:
    """Route the operators through another build of the library for the
    duration of a ``with`` block (the tests' fast-math measurement build)."""

    def __init__(self, other):
        self.other = other

    def __enter__(self):
        global _lib
        lib()
        self.saved, _lib = _lib, self.other
        return self.other

    def __exit__(self, *exc):
        global _lib
        _lib = self.saved
        return False


def exported_symbols():
    """Names declared in include/vorotracing_b200.h (parsed from the header)."""
    import re

    hdr = os.path.join(os.path.dirname(_HERE), "include", "vorotracing_b200.h")
    if not os.path.exists(hdr):
        hdr = os.path.join(_HERE, "vorotracing_b200.h")
    text = open(hdr).read()
    return sorted(set(re.findall(r"\b(vt_[a-z0-9_]+)\s*\(", text)))


def check(status: int, what: str = "") -> None:
    if status != 0:
        msg = lib().vt_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"{what}: error {status}")


def ptr(t):
    """Device/host address of a tensor (None for None or empty tensors)."""
    if t is None:
        return None
    return C.c_void_p(t.data_ptr()) if t.numel() else None


def stream_ptr(device=None):
    import torch

    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)
