"""Fused Adam over the flat per-cell parameter layout (``vt_adam_step``).

The reference optimises four per-cell tensors with torch.optim.Adam
(eps=1e-15) in four learning-rate groups and then clamps the log-density to
at most 30 (vorotracing/trainer.py:258-265, 503-527).  ``CellAdam`` keeps the
parameters, their gradients and both Adam moments in ``GradBucket``-shaped
flat buffers [points 3N | density N | diffuse | specular], so the gradient
all-reduce, the update and the clamp each touch one buffer in one launch.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import check, lib, ptr, stream_ptr
from .shard import GradBucket

GROUPS = ("primal_points", "density", "att_diffuse", "att_specular")


class CellAdam:
    def __init__(self, params: GradBucket, lrs=(1e-4, 1e-2, 1e-2, 1e-2), betas=(0.9, 0.999),
                 eps: float = 1e-15, density_max: float | None = 30.0):
        self.params = params
        self.grads = GradBucket(params.n, params.tex_cols, params.flat.device)
        self.m = torch.zeros_like(params.flat)
        self.v = torch.zeros_like(params.flat)
        self.lrs = list(lrs)
        self.betas = betas
        self.eps = eps
        self.density_max = density_max
        self.t = 0
        n = params.n
        ends = [3 * n, 4 * n, 4 * n + params.tex_cols * n, params.flat.numel()]
        self._ends = (C.c_uint64 * 4)(*ends)

    def set_lr(self, group: str, lr: float):
        self.lrs[GROUPS.index(group)] = float(lr)

    def step(self):
        self.t += 1
        p = self.params.flat
        check(lib().vt_adam_step(ptr(p), ptr(self.grads.flat), ptr(self.m), ptr(self.v),
                                 C.c_uint64(p.numel()), self._ends, (C.c_float * 4)(*self.lrs),
                                 C.c_float(self.betas[0]), C.c_float(self.betas[1]),
                                 C.c_float(self.eps), C.c_uint32(self.t),
                                 C.c_int(1 if self.density_max is not None else -1),
                                 C.c_float(self.density_max or 0.0), stream_ptr(p.device)),
              "vt_adam_step")
