"""Python operator surface with the names and signatures of the reference's
``vorotracing.cuda._wrapper`` (vorotracing/cuda/_wrapper.py:234-307)."""
from __future__ import annotations

from . import _ops


def prefetch_octmap_adj(points, adjacency, offsets):
    """Scene face layout for the inference operators (_wrapper.py:234-237).

    Returns this package's packed face rows (16 bytes per CSR entry) instead of
    the reference's (E+32, 4) half offsets; callers only pass it back to
    trace_octmap_infer / trace_octmap_infer_q8."""
    return _ops.prefetch_faces(points, adjacency, offsets)


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
