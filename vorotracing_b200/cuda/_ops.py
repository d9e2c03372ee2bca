"""Host-side operators over the C ABI, mirroring the reference's ``_C`` ops.

Argument meaning, dtype rules and error messages follow the reference's
validations (vorotracing/cuda/csrc/tracing/validations.h:17-66 and the ASSERTs
of tracing_octmap.cu).  Outputs are allocated with torch on the rays' device
and every kernel is launched on torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _lib
from .._lib import check, lib, ptr, stream_ptr

FACE_ROW_HALVES = 8  # one packed face row = 16 bytes = 8 binary16


def _fail(msg: str):
    raise RuntimeError(msg)


def validate_scene_data(points, attributes, adjacency, offsets):
    """validations.h:17-66, same messages."""
    if points.size(-1) != 3:
        _fail(f"points had dimension {points.size(-1)} along axis -1, expected 3")
    if points.dtype != torch.float32:
        _fail(f"points had dtype {str(points.dtype).replace('torch.', '')}, expected float32")
    if points.device.type != "cuda":
        _fail("points must be on CUDA device")
    n = points.numel() // 3
    if attributes.device.type != "cuda":
        _fail("attributes must be on CUDA device")
    if offsets.dtype != torch.uint32:
        _fail("point_adjacency_offsets must have uint32 dtype")
    if offsets.device.type != "cuda":
        _fail("point_adjacency_offsets must be on CUDA device")
    if offsets.numel() != n + 1:
        _fail("point_adjacency_offsets must have num_points + 1 elements")
    if adjacency.dtype != torch.uint32:
        _fail("point_adjacency must have uint32 dtype")
    if adjacency.device.type != "cuda":
        _fail("point_adjacency must be on CUDA device")


def host_device_ptr(t: torch.Tensor):
    """Device address of a page-locked host tensor (vt_host_device_ptr)."""
    out = C.c_void_p()
    check(lib().vt_host_device_ptr(C.c_void_p(t.data_ptr()), C.byref(out)), "vt_host_device_ptr")
    return out


def _aligned(t: torch.Tensor, align: int) -> torch.Tensor:
    t = t.contiguous()
    if t.numel() and t.data_ptr() % align:
        t = t.clone()
    return t


def prefetch_faces(points, adjacency, offsets) -> torch.Tensor:
    """Packed face rows (E_total + 4, 8) binary16, 16 bytes per CSR entry.

    Replaces trace_vorotracing_prefetch_adj (tracing_octmap.cu:612-640); the
    result is an opaque scene layout consumed by the trace operators."""
    points = points.contiguous()
    adjacency = adjacency.contiguous()
    offsets = offsets.contiguous()
    n = points.size(0)
    e = adjacency.numel()
    rows = int(lib().vt_face_rows(C.c_uint64(e)))
    faces = torch.empty((rows, FACE_ROW_HALVES), dtype=torch.float16, device=points.device)
    err = torch.zeros(1, dtype=torch.int32, device=points.device)
    check(lib().vt_prefetch_adj(ptr(points), C.c_uint32(n), ptr(adjacency), C.c_uint64(e),
                                ptr(offsets), C.c_uint64(e), ptr(faces), C.c_uint64(rows),
                                ptr(err), stream_ptr(points.device)), "vt_prefetch_adj")
    if int(err.item()) != 0:
        _fail("invalid Voronoi adjacency: neighbour index out of range, offsets not monotone "
              "or a cell degree above 65535")
    return faces


def prefetch_adj_diff(points, adjacency, offsets) -> torch.Tensor:
    """The reference's adj_diff, (adjacency_len + 32, 4) binary16 rows
    (trace_vorotracing_prefetch_adj, tracing_octmap.cu:612-640; rows after
    offsets[N] are zero here, uninitialised there).  The packed face rows the
    trace kernels read are written in the same pass and travel with the
    returned tensor (``adj_diff._vt_faces``), so passing it back to the
    inference operators costs nothing extra."""
    points = points.contiguous()
    adjacency = adjacency.contiguous()
    offsets = offsets.contiguous()
    n = points.size(0)
    e = adjacency.numel()
    csr = int(offsets[-1].item()) if offsets.numel() else 0
    L = lib()
    # as many face rows as prefetch_faces makes; rows from offsets[N] on are zero
    faces = torch.empty((int(L.vt_face_rows(C.c_uint64(e))), FACE_ROW_HALVES),
                        dtype=torch.float16, device=points.device)
    drows = int(L.vt_adj_diff_rows(C.c_uint64(e)))
    adj_diff = torch.empty((drows, 4), dtype=torch.float16, device=points.device)
    err = torch.zeros(1, dtype=torch.int32, device=points.device)
    check(L.vt_prefetch_adj_diff(ptr(points), C.c_uint32(n), ptr(adjacency), C.c_uint64(e),
                                 ptr(offsets), C.c_uint64(csr), ptr(faces),
                                 C.c_uint64(faces.size(0)), ptr(adj_diff), C.c_uint64(drows),
                                 ptr(err), stream_ptr(points.device)), "vt_prefetch_adj_diff")
    if int(err.item()) != 0:
        _fail("invalid Voronoi adjacency: neighbour index out of range, offsets not monotone "
              "or a cell degree above 65535")
    adj_diff._vt_faces = faces
    return adj_diff


def _resolve_faces(adjacent_diff, adjacency, points, offsets) -> torch.Tensor:
    """The packed face rows behind an ``adjacent_diff`` argument: the tensor
    itself when it is this package's packed layout, the rows built alongside
    it by prefetch_adj_diff, or (a reference-layout array from elsewhere)
    rows built now from the sites and CSR and kept on that array."""
    if (adjacent_diff.dtype == torch.float16 and adjacent_diff.dim() == 2
            and adjacent_diff.size(1) == 4):
        if adjacent_diff.device != points.device:
            _fail("adjacent_diff must be on the points' device")
        if adjacent_diff.size(0) < adjacency.numel():
            _fail("adjacent_diff must have at least as many rows as point_adjacency")
        faces = getattr(adjacent_diff, "_vt_faces", None)
        if faces is None or faces.device != points.device:
            faces = prefetch_faces(points, adjacency, offsets)
            adjacent_diff._vt_faces = faces
        return faces
    _check_faces(adjacent_diff, adjacency, points)
    return adjacent_diff


def make_scene(points, density, offsets, faces) -> _lib.VtScene:
    return _lib.VtScene(points.data_ptr(), density.data_ptr(), offsets.data_ptr(),
                        faces.data_ptr(), points.size(0), faces.size(0))


def _check_faces(faces, adjacency, points):
    if (faces.dtype != torch.float16 or faces.dim() != 2 or faces.size(1) != FACE_ROW_HALVES
            or faces.size(0) < adjacency.numel()):
        _fail("adjacent_diff must be the (E+32, 4) float16 array returned by "
              "prefetch_octmap_adj, or this package's packed face rows, for the same adjacency")
    if faces.device != points.device:
        _fail("adjacent_diff must be on the points' device")


def _check_err(err):
    if int(err.item()) != 0:
        _fail("trace: invalid start point or ray permutation index (out of range)")


def _res_from(attr: torch.Tensor, channels: int) -> int:
    per = attr.size(1) // channels
    r = int(round(per ** 0.5))
    if r * r * channels != attr.size(1) or r not in (4, 8):
        _fail(f"octahedral texture rows must hold {channels}*R*R values with R in (4, 8), "
              f"got {attr.size(1)}")
    return r


def trace_vorotracing_infer(points, diffuse, specular, density, adjacency, offsets, rays,
                            start_point, adjacent_diff, ray_perm, weight_threshold: float,
                            max_intersections: int, cell_skip_threshold: float,
                            debug: dict | None = None, out=None, host_io: bool = False):
    """fp16 inference (tracing_octmap.cu:642-717).  Returns rgba (..., 4) float16.

    host_io=True (an extension of this package): ``rays`` and ``out`` are
    page-locked host tensors that the kernel reads and writes directly over
    the bus (zero-copy); everything else stays on the device."""
    points = points.contiguous()
    diffuse = _aligned(diffuse, 8)
    specular = _aligned(specular, 8)
    density = density.contiguous()
    adjacency = adjacency.contiguous()
    offsets = offsets.contiguous()
    rays = rays if host_io else _aligned(rays, 8)
    start_point = start_point.contiguous()
    validate_scene_data(points, diffuse, adjacency, offsets)
    if diffuse.dtype != torch.float16:
        _fail("inference kernel requires float16 diffuse")
    if specular.dtype != torch.float16:
        _fail("inference kernel requires float16 specular")
    if density.dtype != torch.float32:
        _fail("density must have float32 dtype")
    if rays.dtype != torch.float32:
        _fail("rays must have float32 dtype")
    if start_point.dtype != torch.uint32:
        _fail("start_point must have uint32 dtype")
    return _infer_common(points, diffuse, specular, density, adjacency, offsets, rays,
                         start_point, adjacent_diff, ray_perm, weight_threshold,
                         max_intersections, cell_skip_threshold, None, debug, out, host_io)


def trace_vorotracing_infer_q8(points, diffuse, specular, density, adjacency, offsets, rays,
                               start_point, adjacent_diff, diff_scale, diff_offset, spec_scale,
                               spec_offset, weight_threshold: float, max_intersections: int,
                               cell_skip_threshold: float, ray_perm=None,
                               debug: dict | None = None, out=None, host_io: bool = False):
    """q8 inference (tracing_octmap.cu:781-854).  Returns rgba (..., 4) float16."""
    points = points.contiguous()
    diffuse = diffuse.contiguous()
    specular = specular.contiguous()
    density = density.contiguous()
    adjacency = adjacency.contiguous()
    offsets = offsets.contiguous()
    rays = rays if host_io else _aligned(rays, 8)
    start_point = start_point.contiguous()
    validate_scene_data(points, diffuse, adjacency, offsets)
    if diffuse.dtype != torch.uint8:
        _fail("q8 inference kernel requires uint8 diffuse")
    if specular.dtype != torch.uint8:
        _fail("q8 inference kernel requires uint8 specular")
    q8 = (float(diff_scale), float(diff_offset), float(spec_scale), float(spec_offset))
    # (N, 4R^2) maps are this package's widened texels (pad_u8x4), read with
    # one 32-bit load per texel; (N, 3R^2) is the reference's layout
    wide = diffuse.dim() == 2 and diffuse.size(1) in (4 * 16, 4 * 64)
    return _infer_common(points, diffuse, specular, density, adjacency, offsets, rays,
                         start_point, adjacent_diff, ray_perm, weight_threshold,
                         max_intersections, cell_skip_threshold, q8, debug, out, host_io,
                         q8_wide=wide)


def _infer_common(points, diffuse, specular, density, adjacency, offsets, rays, start_point,
                  adjacent_diff, ray_perm, wt, max_int, skip, q8, debug, out=None,
                  host_io=False, q8_wide=False):
    if rays.size(-1) != 6:
        _fail("rays must have 6 as the last dimension")
    if host_io:
        if not (rays.is_pinned() and rays.is_contiguous() and rays.data_ptr() % 8 == 0):
            _fail("host_io rays must be contiguous, 8-byte aligned page-locked host memory")
        if out is None or not (out.is_pinned() and out.is_contiguous()):
            _fail("host_io needs a contiguous page-locked host out tensor")
    elif rays.device.type != "cuda":
        _fail("rays must be on CUDA device")
    nr = rays.numel() // 6
    if start_point.numel() != nr:
        _fail("start_point must have the same batch size as rays")
    n = points.size(0)
    if diffuse.size(0) != n or specular.size(0) != n or density.numel() != n:
        _fail("diffuse, specular, density must each have num_points rows")
    faces = _resolve_faces(adjacent_diff, adjacency, points, offsets)
    channels = 3 if (q8 and not q8_wide) else 4
    res = _res_from(diffuse, channels)
    if _res_from(specular, channels) != res:
        _fail("diffuse and specular octahedral resolutions must match")
    perm = None
    if ray_perm is not None and ray_perm.numel():
        perm = ray_perm.contiguous()
        if perm.numel() != nr:
            _fail("ray_perm must be empty or have one entry per ray")
        if perm.dtype not in (torch.int32, torch.uint32):
            _fail("ray_perm must have int32 or uint32 dtype")
    shape = tuple(rays.shape[:-1]) + (4,)
    dev = points.device
    if out is not None:
        if tuple(out.shape) != shape or out.dtype != torch.float16 or not out.is_contiguous():
            _fail("out must be a contiguous float16 tensor of shape rays.shape[:-1] + (4,)")
        rgba = out
    else:
        rgba = torch.empty(shape, dtype=torch.float16, device=dev)
    if host_io:
        rays_p, rgba_p = host_device_ptr(rays), host_device_ptr(rgba)
    else:
        if rgba.device != rays.device:
            _fail("out must be on the rays' device")
        rays_p, rgba_p = ptr(rays), ptr(rgba)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scene = make_scene(points, density, offsets, faces)
    dbg, keep = _debug_struct(debug, nr, n)
    L = lib()
    stream = stream_ptr(dev)
    if q8 is None:
        st = L.vt_trace_infer_f16(C.byref(scene), ptr(diffuse), ptr(specular), C.c_int(res),
                                  rays_p, C.c_uint32(nr), ptr(start_point), ptr(perm),
                                  C.c_float(wt), C.c_uint32(max_int), C.c_float(skip),
                                  rgba_p, dbg, ptr(err), stream)
    else:
        fn = L.vt_trace_infer_q8x4 if q8_wide else L.vt_trace_infer_q8
        st = fn(C.byref(scene), ptr(diffuse), ptr(specular), C.c_int(res),
                                 *[C.c_float(v) for v in q8], rays_p, C.c_uint32(nr),
                                 ptr(start_point), ptr(perm), C.c_float(wt), C.c_uint32(max_int),
                                 C.c_float(skip), rgba_p, dbg, ptr(err), stream)
    check(st, "trace infer")
    if debug is not None or _CHECK_ERRORS:
        _check_err(err)
    del keep
    return rgba


# Reading the device error word forces a host sync; it is skipped on the
# default path of the inference operators (invalid indices then yield zero
# pixels) and always done when diagnostics are requested.
_CHECK_ERRORS = False


def _debug_struct(debug, nr, n_points=0):
    """Allocate the optional per-ray diagnostics requested in ``debug`` (a dict
    that receives the tensors): keys seq_cap (visited-cell sequences), visited
    (per-cell visited / textured flags); stats and num_intersections always."""
    if debug is None:
        return None, None
    dev = torch.device("cuda", torch.cuda.current_device())
    cap = int(debug.get("seq_cap", 0))
    z = lambda *shape, dt=torch.int32: torch.zeros(shape, dtype=dt, device=dev)
    seq = z(nr, cap) if cap else None
    seq_len = z(nr) if cap else None
    stats = z(nr, 4)
    nint = z(nr)
    vis = z(n_points, dt=torch.uint8) if debug.get("visited") else None
    tex = z(n_points, dt=torch.uint8) if debug.get("visited") else None
    debug.update(seq=seq, seq_len=seq_len, stats=stats, num_intersections=nint, visited=vis,
                 textured=tex)
    a = lambda t: None if t is None else t.data_ptr()
    d = _lib.VtDebug(a(seq), cap, a(seq_len), a(stats), a(nint), a(vis), a(tex))
    return C.byref(d), (d, seq, seq_len, stats, nint, vis, tex)


# ---------------------------------------------------------------- BVH

def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class NNBVH:
    """Nearest-site BVH (replaces the reference's cuBQL-backed NNBVH,
    vorotracing/cuda/csrc/utils/nn_bvh.cu:43-109).

    build(points) builds it; query(points, queries) returns the int32 index of
    the nearest site to each query (ties to the lowest index)."""

    def __init__(self):
        self._nodes = None
        self.num_points = 0

    def build(self, points):
        if points.device.type != "cuda":
            _fail("points must be on CUDA")
        points = points.detach().contiguous()
        if points.dtype != torch.float32 or points.dim() != 2 or points.size(1) != 3:
            _fail("points must be a float32 (N, 3) tensor")
        n = points.size(0)
        if n == 0:
            _fail("points must have at least 1 point")
        L = lib()
        nb = int(L.vt_bvh_nodes_bytes(C.c_uint32(n)))
        wb = int(L.vt_bvh_workspace_bytes(C.c_uint32(n)))
        nodes = _ws(nb, points.device)
        ws = _ws(wb, points.device)
        check(L.vt_bvh_build(ptr(points), C.c_uint32(n), ptr(nodes), C.c_uint64(nb), ptr(ws),
                             C.c_uint64(wb), stream_ptr(points.device)), "vt_bvh_build")
        self._nodes = nodes
        self._ws_keep = ws  # freed on the next build; the stream orders reuse
        self.num_points = n

    def query(self, points, queries, hint=None):
        """Nearest site per query (int32).  ``hint``: optional site id(s) (a
        1-element or per-query tensor) believed nearest; it only speeds up the
        search."""
        if self._nodes is None:
            _fail("BVH must be built before querying")
        if queries.device.type != "cuda":
            _fail("queries must be on CUDA")
        points = points.detach().contiguous()
        if points.size(0) != self.num_points:
            _fail("points must be the point set the BVH was built on")
        q = queries.detach().reshape(-1, 3).contiguous().float()
        out = torch.empty(q.size(0), dtype=torch.int32, device=q.device)
        if hint is None:
            check(lib().vt_bvh_query(ptr(self._nodes), ptr(points), C.c_uint32(self.num_points),
                                     ptr(q), C.c_uint32(q.size(0)), ptr(out), None,
                                     stream_ptr(q.device)), "vt_bvh_query")
            return out
        h = hint.detach().reshape(-1).to(device=q.device)
        if h.dtype not in (torch.int32, torch.uint32):
            h = h.to(torch.int32)
        h = h.contiguous()
        if h.numel() not in (1, q.size(0)):
            _fail("hint must hold 1 or one site id per query")
        check(lib().vt_bvh_query_hint(ptr(self._nodes), ptr(points), C.c_uint32(self.num_points),
                                      ptr(q), C.c_uint32(q.size(0)), ptr(h),
                                      C.c_uint32(h.numel()), ptr(out), None,
                                      stream_ptr(q.device)), "vt_bvh_query_hint")
        return out


def nearest_neighbor_bvh(points, queries):
    """One-off build + query (nn_bvh.cu:112-117)."""
    b = NNBVH()
    b.build(points)
    return b.query(points, queries)


# ---------------------------------------------------------------- layout

def morton_codes(points) -> torch.Tensor:
    points = points.detach().contiguous()
    n = points.size(0)
    codes = torch.empty(n, dtype=torch.int64, device=points.device)
    ws = _ws(256, points.device)
    check(lib().vt_morton_codes(ptr(points), C.c_uint32(n), ptr(codes), ptr(ws),
                                stream_ptr(points.device)), "vt_morton_codes")
    return codes


def morton_perm(points):
    """(perm, inv_perm) int64: stable argsort of the sites' Morton codes."""
    points = points.detach().contiguous()
    n = points.size(0)
    dev = points.device
    codes = morton_codes(points)
    wb = int(lib().vt_morton_workspace_bytes(C.c_uint32(n)))
    ws = _ws(wb, dev)
    perm = torch.empty(n, dtype=torch.int32, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    check(lib().vt_morton_perm(ptr(codes), C.c_uint32(n), ptr(perm), ptr(inv), ptr(ws),
                               C.c_uint64(wb), stream_ptr(dev)), "vt_morton_perm")
    return perm, inv


def gather_rows(src: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    src = src.contiguous()
    out = torch.empty_like(src)
    n = src.size(0)
    row = src.numel() // max(n, 1) * src.element_size()
    check(lib().vt_gather_rows(ptr(src), ptr(out), ptr(perm.contiguous()), C.c_uint32(n),
                               C.c_uint32(row), stream_ptr(src.device)), "vt_gather_rows")
    return out


def permute_csr(adjacency, offsets, perm, inv, pad: int = 32):
    n = offsets.numel() - 1
    dev = offsets.device
    wb = int(lib().vt_morton_workspace_bytes(C.c_uint32(n)))
    ws = _ws(wb, dev)
    new_offs = torch.empty(n + 1, dtype=torch.uint32, device=dev)
    new_adj = torch.zeros(adjacency.numel(), dtype=torch.uint32, device=dev)
    check(lib().vt_permute_csr(ptr(offsets.contiguous()), ptr(adjacency.contiguous()),
                               C.c_uint32(n), ptr(perm), ptr(inv), ptr(new_offs), ptr(new_adj),
                               ptr(ws), C.c_uint64(wb), stream_ptr(dev)), "vt_permute_csr")
    return new_adj, new_offs


def tile_perm(H: int, W: int, TH: int = 4, TW: int = 8, device=None) -> torch.Tensor:
    dev = device or torch.device("cuda", torch.cuda.current_device())
    out = torch.empty(H * W, dtype=torch.int32, device=dev)
    check(lib().vt_tile_perm(C.c_uint32(H), C.c_uint32(W), C.c_uint32(TH), C.c_uint32(TW),
                             ptr(out), stream_ptr(dev)), "vt_tile_perm")
    return out


def pad_f16x4(tex: torch.Tensor) -> torch.Tensor:
    """(N, 3R^2) float32 -> (N, 4R^2) float16 Half4Texel rows."""
    tex = tex.detach().contiguous().float()
    n = tex.size(0)
    out = torch.empty((n, tex.size(1) // 3 * 4), dtype=torch.float16, device=tex.device)
    check(lib().vt_pad_f16x4(ptr(tex), C.c_uint64(tex.numel() // 3), ptr(out),
                             stream_ptr(tex.device)), "vt_pad_f16x4")
    return out


def pad_u8x4(tex: torch.Tensor) -> torch.Tensor:
    """(N, 3R^2) uint8 q8 map -> (N, 4R^2) uint8 with a zero 4th byte per
    texel, the widened layout the q8 trace reads with 32-bit loads."""
    tex = tex.contiguous()
    if tex.dtype != torch.uint8 or tex.dim() != 2 or tex.size(1) % 3:
        _fail("pad_u8x4 expects an (N, 3R^2) uint8 map")
    n, texels = tex.size(0), tex.numel() // 3
    out = torch.empty((n, tex.size(1) // 3 * 4), dtype=torch.uint8, device=tex.device)
    check(lib().vt_pad_u8x4(ptr(tex), C.c_uint64(texels), ptr(out), stream_ptr(tex.device)),
          "vt_pad_u8x4")
    return out


def quantize_u8(tex: torch.Tensor):
    """Global min/max uint8 quantisation -> (q, scale, offset) as Python floats."""
    tex = tex.detach().contiguous().float()
    mm = torch.empty(2, dtype=torch.float32, device=tex.device)
    ws = _ws(256, tex.device)
    check(lib().vt_minmax_f32(ptr(tex), C.c_uint64(tex.numel()), C.c_int(1), ptr(ws), ptr(mm),
                              stream_ptr(tex.device)), "vt_minmax_f32")
    vmin, vmax = (float(v) for v in mm.cpu())
    scale = (vmax - vmin) / 255.0
    q = torch.empty(tex.shape, dtype=torch.uint8, device=tex.device)
    check(lib().vt_quantize_u8(ptr(tex), C.c_uint64(tex.numel()), C.c_float(scale),
                               C.c_float(vmin), ptr(q), stream_ptr(tex.device)), "vt_quantize_u8")
    return q, scale, vmin


# ---------------------------------------------------------------- training

def _attr_half(diffuse) -> int:
    if diffuse.dtype == torch.float32:
        return 0
    if diffuse.dtype == torch.float16:
        return 1
    _fail("Unsupported color dtype. Only float32 and float16 are supported.")


def _train_checks(points, diffuse, specular, density, adjacency, offsets, rays, start_point):
    validate_scene_data(points, diffuse, adjacency, offsets)
    n = points.size(0)
    if diffuse.dtype != specular.dtype:
        _fail("diffuse and specular must have the same dtype")
    if not (diffuse.size(0) == specular.size(0) == density.size(0) == n):
        _fail("diffuse, specular, density must each have num_points rows")
    if density.dtype != torch.float32:
        _fail("density must have float32 dtype")
    if rays.size(-1) != 6:
        _fail("rays must have 6 as the last dimension")
    if rays.dtype != torch.float32:
        _fail("rays must have float32 dtype")
    if rays.device.type != "cuda":
        _fail("rays must be on CUDA device")
    nr = rays.numel() // 6
    if start_point.numel() != nr:
        _fail("start_point must have the same batch size as rays")
    if start_point.dtype != torch.uint32:
        _fail("start_point must have uint32 dtype")
    if start_point.device.type != "cuda":
        _fail("start_point must be on CUDA device")
    return nr


class PathRecord:
    """Per-ray walk record written by the training forward and replayed by
    the backward (vt_path): ``steps`` (cap, num_rays, 4) 32-bit words per
    step {cell id, r, g, b as float32 bits}, slot-major; ``len`` (num_rays,)
    uint32 (bit 31: the backward walks the ray itself).  cap * num_rays * 16
    bytes of device memory; rays longer than ``cap`` steps resume the face
    scan after the stored prefix."""

    def __init__(self, num_rays: int, cap: int, device):
        self.cap = int(cap)
        self.num_rays = int(num_rays)
        self.steps = torch.empty((self.cap, self.num_rays, 4), dtype=torch.int32, device=device)
        self.len = torch.empty(self.num_rays, dtype=torch.uint32, device=device)

    @property
    def cells(self) -> torch.Tensor:
        """(cap, num_rays) uint32 cell entered at each step."""
        return self.steps[..., 0].view(torch.uint32)

    @property
    def colors(self) -> torch.Tensor:
        """(cap, num_rays, 3) float32 colour of the segment integrated at each step."""
        return self.steps[..., 1:].view(torch.float32)

    def struct(self, nr: int):
        if nr != self.num_rays:
            _fail("path record was made for a different number of rays")
        return _lib.VtPath(self.steps.data_ptr(), self.cap, self.len.data_ptr())


def _path_arg(path, nr):
    return None if path is None else C.byref(path.struct(nr))


def trace_vorotracing_fwd(points, diffuse, specular, density, adjacency, offsets, rays,
                          start_point, depth_quantiles, weight_threshold: float,
                          max_intersections: int, return_contribution: bool, faces=None,
                          debug: dict | None = None, path: PathRecord | None = None):
    """Training forward (tracing_octmap.cu:355-546).  Returns the reference's
    9-tuple (rgba, depth, depth_indices, contribution, num_intersections,
    distortion, W_total, S_total, t_far); depth / depth_indices /
    contribution are None when not requested.  ``path``: a PathRecord to
    fill for the backward."""
    points, diffuse, specular = points.contiguous(), diffuse.contiguous(), specular.contiguous()
    density, adjacency, offsets = density.contiguous(), adjacency.contiguous(), offsets.contiguous()
    rays, start_point = _aligned(rays, 8), start_point.contiguous()
    nr = _train_checks(points, diffuse, specular, density, adjacency, offsets, rays, start_point)
    half = _attr_half(diffuse)
    res = _res_from(diffuse, 3)
    if _res_from(specular, 3) != res:
        _fail("diffuse and specular octahedral resolutions must match")
    dev = rays.device
    lead = tuple(rays.shape[:-1])
    K = 0
    dq = None
    if depth_quantiles is not None:
        dq = depth_quantiles.contiguous()
        K = dq.size(-1)
        if dq.dtype != torch.float32:
            _fail("depth_quantiles must have float32 dtype")
        if dq.device.type != "cuda":
            _fail("depth_quantiles must be on CUDA device")
        if K == 0 or dq.numel() // K != nr:
            _fail("depth_quantiles must have the same batch size as rays")
    rgba = torch.empty(lead + (4,), dtype=diffuse.dtype, device=dev)
    n_int = torch.empty(lead + (1,), dtype=torch.uint32, device=dev)
    contrib = (torch.zeros((points.size(0), 1), dtype=diffuse.dtype, device=dev)
               if return_contribution else None)
    depth = depth_idx = None
    if dq is not None:
        depth = torch.zeros(lead + (K,), dtype=torch.float32, device=dev)
        depth_idx = torch.zeros(lead + (K,), dtype=torch.uint32, device=dev)
    f32 = lambda: torch.empty(lead + (1,), dtype=torch.float32, device=dev)
    dist, W, S, tfar = f32(), f32(), f32(), f32()
    if faces is None:
        faces = prefetch_faces(points, adjacency, offsets)
    scene = make_scene(points, density, offsets, faces)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dbg, keep = _debug_struct(debug, nr, points.size(0))
    check(lib().vt_trace_fwd(C.byref(scene), C.c_int(half), ptr(diffuse), ptr(specular),
                             C.c_int(res), ptr(rays), C.c_uint32(nr), ptr(start_point),
                             C.c_uint32(K), ptr(dq), C.c_float(weight_threshold),
                             C.c_uint32(max_intersections), ptr(rgba), ptr(depth), ptr(depth_idx),
                             ptr(n_int), ptr(contrib), ptr(dist), ptr(W), ptr(S), ptr(tfar), dbg,
                             _path_arg(path, nr), ptr(err), stream_ptr(dev)), "vt_trace_fwd")
    if debug is not None or _CHECK_ERRORS:
        _check_err(err)
    del keep
    return rgba, depth, depth_idx, contrib, n_int, dist, W, S, tfar


def trace_vorotracing_bwd(points, diffuse, specular, density, adjacency, offsets, rays,
                          start_point, rgb_out, rgb_grad_in, depth_quantiles, depth_indices,
                          depth_grad, ray_error, contribution_alpha_grad: float, distortion,
                          distortion_grad, W_total, S_total, t_far, weight_threshold: float,
                          max_intersections: int, faces=None, grads=None,
                          vector_atomics: bool = True, path: PathRecord | None = None,
                          accumulate: bool = True, workspace: torch.Tensor | None = None,
                          keep_workspace: bool = False):
    """Training backward (tracing_octmap.cu:860-1103).  Gradients go to new
    tensors, or into ``grads`` = (points, diffuse, specular, density) when
    given: added to them, or (``accumulate=False``) overwriting them, which
    spares the caller zeroing them.  Returns the reference's 6-tuple (points_grad, diffuse_grad, specular_grad, density_grad, ray_grad,
    point_error); ray_grad is allocated and never written, as in the
    reference; point_error is None unless ray_error is given.  ``path``: the
    PathRecord filled by the forward of the same inputs (the walk then skips
    the face scan of the recorded steps; results are unchanged).
    ``workspace``: a caller-owned uint8 device tensor of at least
    vt_trace_bwd_workspace_bytes (e.g. one mapped by the other ranks);
    ``keep_workspace`` (with grads, accumulate=False): leave the texel and
    site sums in it for shard.PeerGradReducer instead of writing them to
    ``grads`` (density is written)."""
    points, diffuse, specular = points.contiguous(), diffuse.contiguous(), specular.contiguous()
    density, adjacency, offsets = density.contiguous(), adjacency.contiguous(), offsets.contiguous()
    rays, start_point = _aligned(rays, 8), start_point.contiguous()
    nr = _train_checks(points, diffuse, specular, density, adjacency, offsets, rays, start_point)
    half = _attr_half(diffuse)
    res = _res_from(diffuse, 3)
    dev = rays.device
    g = rgb_grad_in.contiguous()
    if g.size(-1) != 4:
        _fail("rgb_grad_in must have 4 as the last dimension")
    if g.dtype != diffuse.dtype:
        _fail("rgb_grad_in must have the same dtype as diffuse/specular")
    if g.device.type != "cuda":
        _fail("rgb_grad_in must be on CUDA device")
    if g.numel() // 4 != nr:
        _fail("rgb_grad_in must have the same batch size as rays")
    rgb_out = rgb_out.contiguous()
    K = 0
    dq = di = dg = None
    if depth_quantiles is not None:
        dq = depth_quantiles.contiguous()
        K = dq.size(-1)
        if dq.dtype != torch.float32:
            _fail("depth_quantiles must have float32 dtype")
        if dq.numel() != nr * K:
            _fail("depth_quantiles must have the same batch size as rays")
        if depth_grad is None:
            _fail("depth_grad must be provided if depth_quantiles is provided")
        di = depth_indices.contiguous()
        if di.dtype != torch.uint32:
            _fail("depth_indices must have uint32 dtype")
        if di.numel() != nr * K:
            _fail("depth_indices must have the same batch size as rays")
        dg = depth_grad.contiguous()
        if dg.size(-1) != K:
            _fail("depth_grad must have the same number of depth quantiles as depth_quantiles")
        if dg.dtype != torch.float32:
            _fail("depth_grad must have float32 dtype")
        if dg.numel() != nr * K:
            _fail("depth_grad must have the same batch size as rays")
    perr = re = None
    n = points.size(0)
    # the kernels overwrite the outputs when they accumulate in the workspace
    overwrite = bool(vector_atomics) and (grads is None or not accumulate)
    if ray_error is not None:
        re = ray_error.contiguous()
        if re.dtype != diffuse.dtype:
            _fail("ray_error must have the same dtype as diffuse/specular")
        if re.numel() != nr:
            _fail("ray_error must have the same batch size as rays")
        perr = (torch.empty if overwrite else torch.zeros)((n, 1), dtype=diffuse.dtype, device=dev)
    ts = {}
    for name, t in (("W_total", W_total), ("S_total", S_total), ("t_far", t_far),
                    ("distortion", distortion)):
        t = t.contiguous()
        if t.dtype != torch.float32:
            _fail(f"{name} must have float32 dtype")
        if t.numel() != nr:
            _fail(f"{name} must have the same batch size as rays")
        ts[name] = t
    dgr = None
    if distortion_grad is not None:
        dgr = distortion_grad.contiguous()
        if dgr.dtype != torch.float32:
            _fail("distortion_grad must have float32 dtype")
        if dgr.numel() != nr:
            _fail("distortion_grad must have the same batch size as rays")
    if grads is None:
        alloc = torch.empty_like if overwrite else torch.zeros_like
        diffuse_grad = alloc(diffuse)
        specular_grad = alloc(specular)
        density_grad = alloc(density, dtype=torch.float32)
        points_grad = alloc(points, dtype=torch.float32).reshape(n, 3)
    else:
        # caller-provided (e.g. views of a flat all-reduce bucket)
        points_grad, diffuse_grad, specular_grad, density_grad = grads
        if (points_grad.shape != (n, 3) or points_grad.dtype != torch.float32
                or diffuse_grad.shape != diffuse.shape or diffuse_grad.dtype != diffuse.dtype
                or specular_grad.shape != specular.shape
                or specular_grad.dtype != specular.dtype or density_grad.numel() != n
                or density_grad.dtype != torch.float32
                or not all(t.is_contiguous() for t in grads)):
            _fail("grads must be contiguous (points (N,3) f32, diffuse / specular like the "
                  "attributes, density (N,) f32)")
        if not accumulate and not overwrite:
            for t in grads:
                t.zero_()
    ray_grad = torch.empty_like(rays)
    if faces is None:
        faces = prefetch_faces(points, adjacency, offsets)
    scene = make_scene(points, density, offsets, faces)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws, wsb = None, 0
    if keep_workspace and (not vector_atomics or not overwrite or workspace is None
                           or ray_error is not None or half):
        _fail("keep_workspace needs fp32 attributes, vector_atomics, accumulate=False, a caller "
              "workspace and no ray_error")
    if vector_atomics:
        wsb = int(lib().vt_trace_bwd_workspace_bytes(C.c_uint32(n), C.c_int(res)))
        if workspace is not None:
            if (workspace.dtype != torch.uint8 or workspace.numel() < wsb
                    or workspace.device != dev or workspace.data_ptr() % 256):
                _fail(f"workspace must be a 256-byte aligned uint8 tensor of >= {wsb} bytes on "
                      "the rays' device")
            ws, wsb = workspace, workspace.numel()
        else:
            ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    check(lib().vt_trace_bwd(C.byref(scene), C.c_int(half), ptr(diffuse), ptr(specular),
                             C.c_int(res), ptr(rays), C.c_uint32(nr), ptr(start_point),
                             C.c_uint32(K), ptr(dq), ptr(di), ptr(rgb_out), ptr(g), ptr(dg),
                             ptr(re), C.c_float(contribution_alpha_grad),
                             ptr(ts["distortion"]), ptr(dgr), ptr(ts["W_total"]),
                             ptr(ts["S_total"]), C.c_float(weight_threshold),
                             C.c_uint32(max_intersections), ptr(points_grad), ptr(diffuse_grad),
                             ptr(specular_grad), ptr(density_grad), ptr(perr), ptr(ws),
                             C.c_uint64(wsb), _path_arg(path, nr),
                             C.c_uint32((1 if overwrite else 0) | (2 if keep_workspace else 0)),
                             ptr(err), stream_ptr(dev)),
          "vt_trace_bwd")
    if _CHECK_ERRORS:
        _check_err(err)
    return points_grad, diffuse_grad, specular_grad, density_grad, ray_grad, perr


# ---------------------------------------------------------------- Voronoi adjacency

def build_voronoi_adjacency(points, *, debug: bool = False, initial_guesses=None,
                            initial_guesses_offsets=None, chunk_padding: int = 32):
    """Voronoi CSR adjacency of the sites on the GPU (the reference's adapter
    around paragram, vorotracing/cuda/__init__.py:16-46): returns (adjacency
    uint32 with ``chunk_padding`` zero entries at the tail, offsets uint32
    (N+1), status int32 tensor [cells left without neighbours]).
    ``initial_guesses`` / ``initial_guesses_offsets`` (a CSR of guessed
    neighbours, e.g. the adjacency before the sites moved) seed the cells'
    clipping instead of the nearest sites; the result does not depend on
    them.  ``debug`` is accepted for signature compatibility."""
    del debug
    pts = points.detach().contiguous()
    if pts.device.type != "cuda" or pts.dtype != torch.float32 or pts.dim() != 2 or pts.size(1) != 3:
        _fail("points must be a float32 (N, 3) CUDA tensor")
    n = pts.size(0)
    seed_a = seed_o = None
    if (initial_guesses is None) != (initial_guesses_offsets is None):
        _fail("initial_guesses and initial_guesses_offsets go together")
    if initial_guesses is not None:
        seed_a = initial_guesses.to(device=pts.device).contiguous()
        seed_o = initial_guesses_offsets.to(device=pts.device).contiguous()
        if seed_o.numel() != n + 1:
            _fail("initial_guesses_offsets must have num_points + 1 entries")
        if seed_a.dtype not in (torch.int32, torch.uint32):
            seed_a = seed_a.to(torch.int32)
        if seed_o.dtype not in (torch.int32, torch.uint32):
            seed_o = seed_o.to(torch.int32)
    L = lib()
    L.vt_voronoi_bytes.restype = C.c_uint64
    wb = int(L.vt_voronoi_bytes(C.c_uint32(n)))
    ws = _ws(wb, pts.device)
    offs = torch.empty(n + 1, dtype=torch.int32, device=pts.device)
    E = C.c_uint64(0)
    bad = C.c_uint32(0)
    stream = stream_ptr(pts.device)
    check(L.vt_voronoi_adjacency(ptr(pts), C.c_uint32(n), ptr(seed_a), ptr(seed_o), ptr(ws),
                                 C.c_uint64(wb), ptr(offs),
                                 C.byref(E), C.byref(bad), stream), "vt_voronoi_adjacency")
    adj = torch.zeros(int(E.value) + chunk_padding, dtype=torch.int32, device=pts.device)
    check(L.vt_voronoi_write(ptr(ws), C.c_uint32(n), ptr(offs), ptr(adj), stream),
          "vt_voronoi_write")
    status = torch.tensor([int(bad.value)], dtype=torch.int32)
    return adj.view(torch.uint32), offs.view(torch.uint32), status
