"""TEST INFRASTRUCTURE: ctypes front end of the CPU oracle (oracle/vto_oracle.c).

The oracle is a CPU restatement of VoroTracing's traversal hot path
(vorotracing/cuda/csrc/tracing/tracing_octmap.cu and ray_integrator_octmap.cuh
in the reference project).  Only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU baseline legs may import this package; the product
(``vorotracing_b200``) never does.

Parity status: pinned by analytic known-answer scenes and by golden vectors
from the reference's own Python layout code; against the reference CUDA
binary, which cannot be compiled here, traversal parity is unpinned.

All arrays are numpy; binary16 data travels as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libvto.so")
_lib = None

ATTR_F32, ATTR_F16, ATTR_F16X4, ATTR_U8 = 0, 1, 2, 3


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (make -f oracle/Makefile)."""
    src = os.path.join(_HERE, "vto_oracle.c")
    hdr = os.path.join(_HERE, "vto_math.h")
    stale = (not os.path.exists(_LIB_PATH)) or max(
        os.path.getmtime(src), os.path.getmtime(hdr)) > os.path.getmtime(_LIB_PATH)
    if force or stale:
        subprocess.check_call(["make", "-s", "-f", os.path.join(_HERE, "Makefile")])
    return _LIB_PATH


class _Scene(C.Structure):
    _fields_ = [
        ("points", C.c_void_p), ("adj", C.c_void_p), ("offs", C.c_void_p),
        ("adj_diff", C.c_void_p), ("density", C.c_void_p),
        ("diffuse", C.c_void_p), ("specular", C.c_void_p),
        ("n_points", C.c_uint32), ("attr", C.c_int32),
        ("res_d", C.c_int32), ("res_s", C.c_int32),
        ("dq_scale", C.c_float), ("dq_offset", C.c_float),
        ("sq_scale", C.c_float), ("sq_offset", C.c_float),
    ]


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.vto_max_threads.restype = C.c_int
    return _lib


def max_threads() -> int:
    return lib().vto_max_threads()


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class Scene:
    """Scene arrays in the reference's own layout (adj_diff = half4 rows).

    attr: ATTR_F32 / ATTR_F16 (N, 3R^2), ATTR_F16X4 (N, 4R^2), ATTR_U8 (N, 3R^2).
    """

    def __init__(self, points, adjacency, offsets, density, diffuse, specular, attr,
                 res_d=None, res_s=None, q8=(1.0, 0.0, 1.0, 0.0)):
        self.points = _c(points, np.float32)
        self.adj = _c(adjacency, np.uint32)
        self.offs = _c(offsets, np.uint32)
        self.density = _c(np.asarray(density).reshape(-1), np.float32)
        dt = {ATTR_F32: np.float32, ATTR_F16: np.uint16, ATTR_F16X4: np.uint16,
              ATTR_U8: np.uint8}[attr]
        if attr in (ATTR_F16, ATTR_F16X4) and np.asarray(diffuse).dtype == np.float16:
            diffuse = np.asarray(diffuse).view(np.uint16)
            specular = np.asarray(specular).view(np.uint16)
        self.diffuse = _c(diffuse, dt)
        self.specular = _c(specular, dt)
        n = self.points.shape[0]
        ch = 4 if attr == ATTR_F16X4 else 3
        if res_d is None:
            res_d = int(round((self.diffuse.size // n // ch) ** 0.5))
        if res_s is None:
            res_s = int(round((self.specular.size // n // ch) ** 0.5))
        self.attr, self.res_d, self.res_s, self.q8 = attr, res_d, res_s, q8
        self.adj_diff = prefetch_adj(self.points, self.adj, self.offs)
        self._s = _Scene(_p(self.points), _p(self.adj), _p(self.offs), _p(self.adj_diff),
                         _p(self.density), _p(self.diffuse), _p(self.specular),
                         n, attr, res_d, res_s, *[float(v) for v in q8])


def prefetch_adj(points, adj, offs, pad_rows: int = 32):
    """Reference prefetch (tracing_octmap.cu:125-149): (E+pad, 4) binary16 bits."""
    points = _c(points, np.float32)
    adj = _c(adj, np.uint32)
    offs = _c(offs, np.uint32)
    rows = int(adj.shape[0]) + pad_rows
    out = np.zeros((rows, 4), np.uint16)
    lib().vto_prefetch_adj(_p(points), C.c_uint32(points.shape[0]), _p(adj), _p(offs), _p(out),
                           C.c_uint64(rows))
    return out


def trace_infer(scene: Scene, rays, start, wt=0.001, max_int=1024, skip=0.0, seq_cap=0,
                threads=0):
    """fp16 / q8 inference.  Returns dict(rgba=float16 (R,4), n, stats, seq, seq_len)."""
    rays = _c(rays, np.float32).reshape(-1, 6)
    start = _c(start, np.uint32).reshape(-1)
    nr = rays.shape[0]
    rgba = np.zeros((nr, 4), np.uint16)
    n = np.zeros(nr, np.uint32)
    stats = np.zeros((nr, 4), np.uint32)
    seq = np.zeros((nr, seq_cap), np.uint32) if seq_cap else None
    seq_len = np.zeros(nr, np.uint32) if seq_cap else None
    lib().vto_trace_infer(C.byref(scene._s), _p(rays), C.c_uint32(nr), _p(start), C.c_float(wt),
                          C.c_uint32(max_int), C.c_float(skip), _p(rgba), _p(n), _p(stats),
                          _p(seq), C.c_uint32(seq_cap), _p(seq_len), C.c_int(threads))
    return dict(rgba=rgba.view(np.float16), n=n, stats=stats, seq=seq, seq_len=seq_len)


def trace_fwd(scene: Scene, rays, start, depth_quantiles=None, wt=0.001, max_int=1024,
              return_contribution=False, seq_cap=0, threads=0):
    """Training forward.  Returns the reference's 9 outputs plus sequences."""
    rays = _c(rays, np.float32).reshape(-1, 6)
    start = _c(start, np.uint32).reshape(-1)
    nr = rays.shape[0]
    K = 0
    dq = None
    if depth_quantiles is not None:
        dq = _c(depth_quantiles, np.float32)
        K = dq.shape[-1]
        dq = dq.reshape(nr, K)
    half = scene.attr == ATTR_F16
    rgba = np.zeros((nr, 4), np.uint16 if half else np.float32)
    qd = np.zeros((nr, max(K, 1)), np.float32)
    qi = np.zeros((nr, max(K, 1)), np.uint32)
    n = np.zeros(nr, np.uint32)
    contrib = np.zeros(scene.points.shape[0], np.float32) if return_contribution else None
    dist, W, S, tf = (np.zeros(nr, np.float32) for _ in range(4))
    seq = np.zeros((nr, seq_cap), np.uint32) if seq_cap else None
    seq_len = np.zeros(nr, np.uint32) if seq_cap else None
    lib().vto_trace_fwd(C.byref(scene._s), _p(rays), C.c_uint32(nr), _p(start), C.c_uint32(K),
                        _p(dq), C.c_float(wt), C.c_uint32(max_int), _p(rgba), _p(qd), _p(qi),
                        _p(n), _p(contrib), _p(dist), _p(W), _p(S), _p(tf), _p(seq),
                        C.c_uint32(seq_cap), _p(seq_len), C.c_int(threads))
    return dict(rgba=rgba.view(np.float16) if half else rgba,
                depth=qd[:, :K], depth_idx=qi[:, :K], contribution=contrib, n=n,
                distortion=dist, W=W, S=S, t_far=tf, seq=seq, seq_len=seq_len)


def trace_bwd(scene: Scene, rays, start, rgba, rgba_grad, depth_quantiles=None,
              depth_idx=None, depth_grad=None, ray_error=None, contribution_alpha_grad=0.0,
              distortion=None, distortion_grad=None, W=None, S=None, t_far=None, wt=0.001,
              max_int=1024, threads=0):
    """Backward.  Returns dict(points, diffuse, specular, density, point_error) in float32."""
    rays = _c(rays, np.float32).reshape(-1, 6)
    start = _c(start, np.uint32).reshape(-1)
    nr = rays.shape[0]
    half = scene.attr == ATTR_F16

    def attr_arr(a):
        if a is None:
            return None
        a = np.asarray(a)
        if half:
            return _c(a.astype(np.float16), np.float16).view(np.uint16)
        return _c(a, np.float32)

    K = 0
    dq = qi = dg = None
    if depth_quantiles is not None:
        dq = _c(depth_quantiles, np.float32)
        K = dq.shape[-1]
        dq = dq.reshape(nr, K)
        qi = _c(depth_idx, np.uint32).reshape(nr, K)
        dg = _c(depth_grad, np.float32).reshape(nr, K)
    f = lambda a: None if a is None else _c(a, np.float32).reshape(-1)
    n = scene.points.shape[0]
    pg = np.zeros((n, 3), np.float32)
    dgr = np.zeros(scene.diffuse.shape, np.float32)
    sgr = np.zeros(scene.specular.shape, np.float32)
    den = np.zeros(n, np.float32)
    perr = np.zeros(n, np.float32) if ray_error is not None else None
    keep = [attr_arr(rgba), attr_arr(rgba_grad), attr_arr(ray_error), f(distortion),
            f(distortion_grad), f(W), f(S), f(t_far)]
    lib().vto_trace_bwd(C.byref(scene._s), _p(rays), C.c_uint32(nr), _p(start), C.c_uint32(K),
                        _p(dq), _p(qi), _p(keep[0]), _p(keep[1]), _p(dg), _p(keep[2]),
                        C.c_float(contribution_alpha_grad), _p(keep[3]), _p(keep[4]),
                        _p(keep[5]), _p(keep[6]), _p(keep[7]),
                        C.c_float(wt), C.c_uint32(max_int), _p(pg), _p(dgr), _p(sgr), _p(den),
                        _p(perr), C.c_int(threads))
    return dict(points=pg, diffuse=dgr, specular=sgr, density=den, point_error=perr)


def nn_query(points, queries, threads=0):
    points = _c(points, np.float32)
    queries = _c(queries, np.float32).reshape(-1, 3)
    out = np.zeros(queries.shape[0], np.int32)
    lib().vto_nn_query(_p(points), C.c_uint32(points.shape[0]), _p(queries),
                       C.c_uint32(queries.shape[0]), _p(out), C.c_int(threads))
    return out


def expf(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().vto_expf_array(_p(x), _p(y), C.c_uint64(x.size))
    return y


def logf(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().vto_logf_array(_p(x), _p(y), C.c_uint64(x.size))
    return y


def f2h(x):
    x = _c(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().vto_f2h_array(_p(x), _p(y), C.c_uint64(x.size))
    return y


# ---------------------------------------------------------------- reference layout helpers

def pad_f16x4(a: np.ndarray, res: int) -> np.ndarray:
    """(N, 3R^2) float -> (N, 4R^2) float16 with a zero 4th channel (the
    reference's _pad_3to4, vorotracing.py:505-512)."""
    n = a.shape[0]
    t = a.reshape(n, res * res, 3).astype(np.float16)
    out = np.zeros((n, res * res, 4), np.float16)
    out[..., :3] = t
    return out.reshape(n, 4 * res * res)


def quantize_u8(a: np.ndarray):
    """The reference's _quantize_to_uint8 (vorotracing.py:495-503) in numpy."""
    vmin = float(a.min())
    vmax = float(a.max())
    scale = (vmax - vmin) / 255.0
    q = np.clip(np.rint((a - np.float32(vmin)) / np.float32(scale)), 0, 255).astype(np.uint8)
    return q, scale, vmin
