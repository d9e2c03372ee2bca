"""Work partitioning across the GPUs of one box (one process per GPU).

Inference (no reference counterpart; the reference is single-GPU): the scene
is replicated and the independent units are views (``view_shard``) or, for a
single large frame, interleaved bands of 4 pixel rows, the height of a 4x8
warp tile (``row_band_shard``).  Neither needs a collective on the data path.

Training: every rank renders its own rays against the same scene, and the
per-cell gradients are summed across ranks with one NCCL all-reduce of a
flat fp32 bucket [points 3N | density N | diffuse 3R^2 N | specular 3R^2 N]
(``GradBucket``).  The backward kernel writes straight into views of the
bucket, so the reduction needs no packing copy.
"""
from __future__ import annotations

import numpy as np
import torch


def view_shard(n_views: int, rank: int, world: int) -> list[int]:
    """Views of this rank, round-robin."""
    return list(range(rank, n_views, world))


def row_band_shard(height: int, rank: int, world: int, band: int = 4) -> np.ndarray:
    """Pixel rows of this rank: bands of ``band`` rows dealt round-robin."""
    rows = np.arange(height)
    return rows[(rows // band) % world == rank]


class GradBucket:
    """Flat gradient buffer with per-parameter views laid out for one all-reduce."""

    def __init__(self, n_points: int, tex_cols: int, device, dtype=torch.float32):
        self.n = n_points
        self.tex_cols = tex_cols
        sizes = [3 * n_points, n_points, tex_cols * n_points, tex_cols * n_points]
        self.flat = torch.zeros(sum(sizes), dtype=dtype, device=device)
        parts = torch.split(self.flat, sizes)
        self.points = parts[0].view(n_points, 3)
        self.density = parts[1].view(n_points, 1)
        self.diffuse = parts[2].view(n_points, tex_cols)
        self.specular = parts[3].view(n_points, tex_cols)

    def views(self):
        return self.points, self.diffuse, self.specular, self.density

    def zero_(self):
        self.flat.zero_()
        return self

    def allreduce_(self, group=None, average: bool = False):
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            if average:
                self.flat.div_(dist.get_world_size(group))
        return self

    @property
    def nbytes(self) -> int:
        return self.flat.numel() * self.flat.element_size()
