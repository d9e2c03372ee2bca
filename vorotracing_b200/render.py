"""Inference-side scene preparation and rendering (the reference's
``VoroTracingInfer``, vorotracing/vorotracing.py:439-683), on this package's
kernels: quantisation / fp16 padding, Morton reordering of cells and CSR,
BVH start-cell lookup, 4x8 warp-tile ray order, and the inference trace."""
from __future__ import annotations

from typing import Literal

import torch

from .cuda import _ops


class InferScene:
    """Renderable scene.

    points (N,3) f32; density (N,1) f32 *activated* density; adjacency / offsets
    uint32 CSR (with tail padding); diffuse / specular (N, 3R^2) f32 logits.
    """

    def __init__(self, points, density, adjacency, offsets, diffuse, specular,
                 quantize: Literal["fp16", "q8"] = "fp16", sort_morton: bool = True):
        dev = points.device
        self.quantize = quantize
        self.primal_points = points.detach().contiguous()
        self.density = density.detach().reshape(-1, 1).contiguous().float()
        self.point_adjacency = adjacency.contiguous()
        self.point_adjacency_offsets = offsets.contiguous()
        if quantize == "q8":
            self.diffuse_q8, self.diff_scale, self.diff_offset = _ops.quantize_u8(diffuse)
            self.specular_q8, self.spec_scale, self.spec_offset = _ops.quantize_u8(specular)
        elif quantize == "fp16":
            self.diffuse_fp16 = _ops.pad_f16x4(diffuse)
            self.specular_fp16 = _ops.pad_f16x4(specular)
        else:
            raise ValueError(f"Invalid quantization method: {quantize}")
        if sort_morton:
            self._reorder_by_morton()
        if quantize == "q8":
            # widened copies (a zero 4th byte per texel) for 32-bit texel loads
            self.diffuse_q8x4 = _ops.pad_u8x4(self.diffuse_q8)
            self.specular_q8x4 = _ops.pad_u8x4(self.specular_q8)
        self.bvh = _ops.NNBVH()
        self.bvh.build(self.primal_points)
        self.adjacent_diff = _ops.prefetch_faces(self.primal_points, self.point_adjacency,
                                                 self.point_adjacency_offsets)
        self._tile_cache = {}
        self.device = dev

    def _reorder_by_morton(self):
        perm, inv = _ops.morton_perm(self.primal_points)
        g = lambda t: _ops.gather_rows(t, perm)
        self.primal_points = g(self.primal_points)
        self.density = g(self.density)
        if self.quantize == "q8":
            self.diffuse_q8, self.specular_q8 = g(self.diffuse_q8), g(self.specular_q8)
        else:
            self.diffuse_fp16, self.specular_fp16 = g(self.diffuse_fp16), g(self.specular_fp16)
        self.point_adjacency, self.point_adjacency_offsets = _ops.permute_csr(
            self.point_adjacency, self.point_adjacency_offsets, perm, inv)
        self.perm = perm

    def tile_perm(self, H: int, W: int) -> torch.Tensor:
        key = (int(H), int(W))
        if key not in self._tile_cache:
            self._tile_cache[key] = _ops.tile_perm(H, W, device=self.primal_points.device)
        return self._tile_cache[key]

    def get_starting_point(self, rays, per_ray: bool = False) -> torch.Tensor:
        """Start cell per ray.  Default: the first ray's origin cell broadcast to
        all rays, as the reference does (vorotracing.py:585-604, pinhole views);
        per_ray=True queries every ray origin (moving or non-pinhole cameras)."""
        lead = rays.shape[:-1]
        flat = rays.reshape(-1, rays.shape[-1])
        if per_ray:
            # the first origin's cell bounds every ray's search (origins of a
            # moving or thick-lens camera stay close together)
            first = self.bvh.query(self.primal_points, flat[:1, :3])
            idx = self.bvh.query(self.primal_points, flat[:, :3], hint=first)
            return idx.view(torch.uint32).reshape(lead)
        idx = self.bvh.query(self.primal_points, flat[:1, :3])
        return idx.expand(flat.shape[0]).reshape(lead).contiguous().view(torch.uint32)

    def render(self, rays, start_point=None, weight_threshold=0.001, max_intersections=1024,
               cell_skip_threshold=0.0, use_warp_perm: bool = True, per_ray_start: bool = False,
               debug=None, out=None, host_io: bool = False):
        ray_perm = None
        if use_warp_perm and rays.dim() == 3 and rays.shape[-1] == 6:
            ray_perm = self.tile_perm(rays.shape[0], rays.shape[1])
        if start_point is None:
            start_point = self.get_starting_point(rays, per_ray_start)
        else:
            start_point = torch.broadcast_to(start_point, rays.shape[:-1])
        if self.quantize == "q8":
            return _ops.trace_vorotracing_infer_q8(
                self.primal_points, self.diffuse_q8x4, self.specular_q8x4, self.density,
                self.point_adjacency, self.point_adjacency_offsets, rays, start_point,
                self.adjacent_diff, self.diff_scale, self.diff_offset, self.spec_scale,
                self.spec_offset, weight_threshold, max_intersections, cell_skip_threshold,
                ray_perm=ray_perm, debug=debug, out=out, host_io=host_io)
        return _ops.trace_vorotracing_infer(
            self.primal_points, self.diffuse_fp16, self.specular_fp16, self.density,
            self.point_adjacency, self.point_adjacency_offsets, rays, start_point,
            self.adjacent_diff, ray_perm, weight_threshold, max_intersections,
            cell_skip_threshold, debug=debug, out=out, host_io=host_io)

    def render_depth(self, rays, mode: str = "mean", n: int = 8, threshold: float = 0.5,
                     start_point=None, weight_threshold=0.001, max_intersections=1024,
                     use_warp_perm: bool = True, per_ray_start: bool = False,
                     thresholds=None):
        """Depth image (the viewer's depth modes, vorotracing/viewer.py:414-433).

        mode "mean": mean of the depths at n transmittance levels
        linspace(1 - 1/(2n), 1/(2n), n) over the positive ones; mode
        "quantile": depth where transmittance falls below ``threshold``.
        ``thresholds`` (K,) overrides the levels of either mode.
        -1 where undefined.  Returns float32 of shape rays.shape[:-1]."""
        import ctypes as C

        from ._lib import check, lib, ptr, stream_ptr

        dev = rays.device
        if mode == "mean":
            thr = torch.linspace(1 - 1 / (2 * n), 1 / (2 * n), n, device=dev)
            m = 1
        elif mode == "quantile":
            thr = torch.full((1,), float(threshold), device=dev)
            m = 0
        else:
            raise ValueError(f"unknown depth mode {mode!r}")
        if thresholds is not None:
            thr = torch.as_tensor(thresholds, dtype=torch.float32, device=dev).reshape(-1)
        rays_c = rays.contiguous()
        ray_perm = None
        if use_warp_perm and rays.dim() == 3 and rays.shape[-1] == 6:
            ray_perm = self.tile_perm(rays.shape[0], rays.shape[1])
        if start_point is None:
            start_point = self.get_starting_point(rays_c, per_ray_start)
        start_point = torch.broadcast_to(start_point, rays.shape[:-1]).contiguous()
        out = torch.empty(rays.shape[:-1], dtype=torch.float32, device=dev)
        scene = _ops.make_scene(self.primal_points, self.density, self.point_adjacency_offsets,
                                self.adjacent_diff)
        check(lib().vt_trace_depth(C.byref(scene), ptr(rays_c), C.c_uint32(rays.numel() // 6),
                                   ptr(start_point), ptr(ray_perm), ptr(thr),
                                   C.c_uint32(thr.numel()), C.c_int(m),
                                   C.c_float(weight_threshold), C.c_uint32(max_intersections),
                                   ptr(out), None, stream_ptr(dev)), "vt_trace_depth")
        return out

    def render_host(self, rays_host: torch.Tensor, out_host: torch.Tensor | None = None,
                    transfer: Literal["zero_copy", "bands"] = "zero_copy", bands: int = 4,
                    sync: bool = True, start_point=None, per_ray_start: bool = False,
                    **kw) -> torch.Tensor:
        """End-to-end render of host rays: rays in, float16 rgba back in host
        memory.  Returns the host tensor.

        transfer="zero_copy" (default; ``rays_host`` must be page-locked): one
        trace launch reads each ray from host memory over the bus and writes
        its pixel straight back, so the 24 + 8 bytes per ray cross the bus
        while the walk runs instead of before and after it.
        transfer="bands": copies in row bands (heights a multiple of 4, so the
        4x8 warp tiles stay whole) on two copy streams, band i+1's upload and
        band i-1's download overlapping band i's trace.
        Rays are independent, so both equal the device render bit for bit.
        The start cell is the frame's first ray's cell (the reference's
        broadcast, vorotracing.py:585-604) unless ``start_point`` or
        ``per_ray_start`` is given; the first ray's origin is the only part
        copied ahead.  With ``sync=False`` the call returns once the work is
        queued and the current stream is ordered after it, so an event
        recorded there afterwards marks completion; rays that had to be
        staged into page-locked memory are kept alive by the scene until the
        trace that reads them has finished."""
        dev = self.primal_points.device
        cur = torch.cuda.current_stream(dev)
        self._staged = [(t, e) for t, e in getattr(self, "_staged", []) if not e.query()]
        if out_host is None:
            out_host = torch.empty(tuple(rays_host.shape[:-1]) + (4,), dtype=torch.float16,
                                   pin_memory=True)
        if transfer == "zero_copy":
            staged = False
            if not (rays_host.is_pinned() and rays_host.is_contiguous()
                    and rays_host.data_ptr() % 8 == 0):
                rays_host = rays_host.contiguous().pin_memory()
                staged = True
            if not (out_host.is_pinned() and out_host.is_contiguous()):
                # the kernel writes page-locked memory only: render into a
                # page-locked buffer and copy into the caller's
                tmp = self.render_host(rays_host, None, transfer, bands, True, start_point,
                                       per_ray_start, **kw)
                out_host.copy_(tmp)
                return out_host
            if per_ray_start and start_point is None:
                rays_dev = rays_host.to(dev, non_blocking=True)
                start_point = self.get_starting_point(rays_dev, per_ray=True)
            elif start_point is None:
                first = rays_host.reshape(-1, rays_host.shape[-1])[:1].to(dev, non_blocking=True)
                start_point = self.get_starting_point(first).reshape(
                    (1,) * (rays_host.dim() - 1))
            self.render(rays_host, start_point=start_point, out=out_host, host_io=True, **kw)
            if sync:
                cur.synchronize()
            elif staged:
                # the kernel reads the staging buffer through its raw address,
                # which torch's host allocator does not track: hold the buffer
                # until an event behind the trace has completed, or the
                # allocator could hand it to the next pin_memory() mid-trace
                done = torch.cuda.Event()
                done.record(cur)
                self._staged.append((rays_host, done))
            return out_host
        if transfer != "bands":
            raise ValueError(f"unknown transfer mode {transfer!r}")
        if rays_host.dim() != 3 or bands <= 1 or rays_host.shape[0] < 8:
            rays = rays_host.to(dev, non_blocking=True)
            rgba = self.render(rays, start_point=start_point, per_ray_start=per_ray_start, **kw)
            out_host.copy_(rgba, non_blocking=True)
            if sync:
                cur.synchronize()
            return out_host
        H = rays_host.shape[0]
        bh = -(-H // (bands * 4)) * 4
        cuts = [(y, min(y + bh, H)) for y in range(0, H, bh)]
        key = (tuple(rays_host.shape), dev)
        if getattr(self, "_host_key", None) != key:
            self._host_key = key
            self._host_rays = torch.empty(rays_host.shape, dtype=torch.float32, device=dev)
            self._h2d = torch.cuda.Stream(dev)
            self._d2h = torch.cuda.Stream(dev)
        rays_dev, h2d, d2h = self._host_rays, self._h2d, self._d2h
        h2d.wait_stream(cur)  # the previous call's traces may still read rays_dev
        d2h.wait_stream(cur)
        ev_in = []
        with torch.cuda.stream(h2d):
            for y0, y1 in cuts:
                rays_dev[y0:y1].copy_(rays_host[y0:y1], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d)
                ev_in.append(e)
        keep = []
        for (y0, y1), e in zip(cuts, ev_in):
            cur.wait_event(e)
            band = rays_dev[y0:y1]
            if start_point is not None:
                sp = torch.broadcast_to(start_point, rays_host.shape[:-1])[y0:y1]
            elif per_ray_start:
                sp = self.get_starting_point(band, per_ray=True)
            else:
                if y0 == 0:
                    first = self.get_starting_point(band[:1, :1])
                sp = first.reshape(1, 1).expand(y1 - y0, band.shape[1])
            rgba = self.render(band, start_point=sp, **kw)
            done = torch.cuda.Event()
            done.record(cur)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                out_host[y0:y1].copy_(rgba, non_blocking=True)
            keep.append(rgba)
        cur.wait_stream(d2h)
        for t in keep:  # freed on the current stream only after the downloads
            t.record_stream(d2h)
        if sync:
            cur.synchronize()
        return out_host
