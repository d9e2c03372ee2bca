"""Python operator surface with the names and signatures of the reference's
``vorotracing.cuda._wrapper`` (vorotracing/cuda/_wrapper.py:234-307)."""
from __future__ import annotations

import torch

from . import _ops


class ErrorBox:
    """Side channel of TraceVoroTracing (_wrapper.py:15-19): set ray_error
    before backward to get per-cell point_error; cell_distortion_gate (N,1)
    routes the distortion gradient of density through a per-cell gate."""

    def __init__(self):
        self.ray_error = None
        self.point_error = None
        self.cell_distortion_gate = None


class TraceVoroTracing(torch.autograd.Function):
    """Differentiable render (_wrapper.py:22-231).

    forward(points, diffuse, specular, density, adjacency, offsets, rays,
    start_point, depth_quantiles, weight_threshold, max_intersections,
    return_contribution) -> (rgba, depth, contribution, num_intersections,
    errbox, distortion).  Gradients flow to the first four inputs.  The packed
    face rows built in forward are reused by backward (the sites cannot change
    in between), where the reference rebuilds its adj_diff on every call.

    The forward also records each ray's first ``path_cap`` steps (cell and
    segment colour, ``path_cap`` * 16 bytes per ray, held until backward; 384 covers all
    but a handful of the rays of 3M-site scenes) so
    that the backward enters them without scanning faces or re-reading
    texels; set ``path_cap = 0`` to re-walk instead.  Gradients are the same
    either way."""

    path_cap = 384

    @staticmethod
    def forward(ctx, _points, _diffuse, _specular, _density, _point_adjacency,
                _point_adjacency_offsets, rays, start_point, depth_quantiles,
                weight_threshold: float, max_intersections: int, return_contribution: bool):
        faces = _ops.prefetch_faces(_points, _point_adjacency, _point_adjacency_offsets)
        cap = min(int(TraceVoroTracing.path_cap), int(max_intersections))
        path = _ops.PathRecord(rays.numel() // 6, cap, rays.device) if cap > 0 else None
        (rgba, depth, depth_indices, contribution, num_intersections, distortion, W_total,
         S_total, t_far) = _ops.trace_vorotracing_fwd(
            _points, _diffuse, _specular, _density, _point_adjacency, _point_adjacency_offsets,
            rays, start_point, depth_quantiles, weight_threshold, max_intersections,
            return_contribution, faces=faces, path=path)
        ctx.path = path
        ctx.args = (_points, _diffuse, _specular, _density, _point_adjacency,
                    _point_adjacency_offsets, rays, start_point)
        ctx.depth_quantiles = depth_quantiles
        ctx.weight_threshold = weight_threshold
        ctx.max_intersections = max_intersections
        ctx.faces = faces
        ctx.rgba = rgba
        ctx.depth_indices = depth_indices
        ctx.distortion, ctx.W_total, ctx.S_total, ctx.t_far = distortion, W_total, S_total, t_far
        errbox = ErrorBox()
        ctx.errbox = errbox
        return rgba, depth, contribution, num_intersections, errbox, distortion

    @staticmethod
    def backward(ctx, grad_rgba, grad_depth, grad_contribution, grad_num_intersections,
                 errbox_grad, grad_distortion):
        contribution_alpha_grad = 0.0
        if grad_contribution is not None:
            contribution_alpha_grad = float(grad_contribution.detach().abs().max().item())
        if grad_rgba is None:
            grad_rgba = torch.zeros_like(ctx.rgba)

        def _bwd(g_rgba, g_depth, ray_error, contrib, g_dist):
            return _ops.trace_vorotracing_bwd(
                *ctx.args, ctx.rgba, g_rgba, ctx.depth_quantiles, ctx.depth_indices,
                g_depth if ctx.depth_quantiles is not None else None, ray_error, contrib,
                ctx.distortion, g_dist, ctx.W_total, ctx.S_total, ctx.t_far,
                ctx.weight_threshold, ctx.max_intersections, faces=ctx.faces, path=ctx.path)

        if ctx.depth_quantiles is not None and grad_depth is None:
            grad_depth = torch.zeros(ctx.depth_indices.shape, dtype=torch.float32,
                                     device=ctx.rgba.device)
        cell_gate = getattr(ctx.errbox, "cell_distortion_gate", None)
        if cell_gate is not None and grad_distortion is not None:
            res_d = _bwd(torch.zeros_like(grad_rgba), None if ctx.depth_quantiles is None
                         else torch.zeros_like(grad_depth), None, 0.0, grad_distortion)
            density_grad_dist = res_d[3]
            (points_grad, diffuse_grad, specular_grad, density_grad, _ray_grad,
             point_error) = _bwd(grad_rgba, grad_depth, ctx.errbox.ray_error,
                                 contribution_alpha_grad, torch.zeros_like(grad_distortion))
            torch.nan_to_num(density_grad_dist, nan=0.0, posinf=0.0, neginf=0.0,
                             out=density_grad_dist)
            density_grad = density_grad + cell_gate.reshape_as(density_grad) * density_grad_dist
        else:
            (points_grad, diffuse_grad, specular_grad, density_grad, _ray_grad,
             point_error) = _bwd(grad_rgba, grad_depth, ctx.errbox.ray_error,
                                 contribution_alpha_grad, grad_distortion)
        ctx.errbox.point_error = point_error
        for t in (points_grad, diffuse_grad, specular_grad, density_grad):
            torch.nan_to_num(t, nan=0.0, posinf=0.0, neginf=0.0, out=t)
        del ctx.args, ctx.faces, ctx.path, ctx.rgba, ctx.distortion, ctx.W_total, ctx.S_total, ctx.t_far
        return (points_grad, diffuse_grad, specular_grad, density_grad, None, None, None, None,
                None, None, None, None)


def prefetch_octmap_adj(points, adjacency, offsets):
    """Neighbour differences for the inference operators (_wrapper.py:234-237).

    Returns the reference's array: (len(adjacency) + 32, 4) float16 rows
    half(points[adj[e]] - points[i]), 0 (tracing_octmap.cu:612-640), which
    callers may keep and export (scripts/export_for_viewer.py writes it into
    V3 .foam files).  The packed face rows the kernels read are built in the
    same pass and ride along on the returned tensor."""
    return _ops.prefetch_adj_diff(points, adjacency, offsets)


def trace_octmap_infer(points, diffuse_fp16, specular_fp16, density, adjacency, offsets, rays,
                       start_point, adjacent_diff, ray_perm, weight_threshold=0.001,
                       max_intersections=1024, cell_skip_threshold=0.0):
    """fp16 inference render (_wrapper.py:240-269)."""
    return _ops.trace_vorotracing_infer(points, diffuse_fp16, specular_fp16, density, adjacency,
                                        offsets, rays, start_point, adjacent_diff, ray_perm,
                                        weight_threshold, max_intersections, cell_skip_threshold)


def trace_octmap_infer_q8(points, diffuse_q8, specular_q8, density, adjacency, offsets, rays,
                          start_point, adjacent_diff, diff_scale, diff_offset, spec_scale,
                          spec_offset, weight_threshold=0.001, max_intersections=1024,
                          cell_skip_threshold=0.0):
    """q8 inference render (_wrapper.py:272-307)."""
    return _ops.trace_vorotracing_infer_q8(points, diffuse_q8, specular_q8, density, adjacency,
                                           offsets, rays, start_point, adjacent_diff, diff_scale,
                                           diff_offset, spec_scale, spec_offset, weight_threshold,
                                           max_intersections, cell_skip_threshold)
