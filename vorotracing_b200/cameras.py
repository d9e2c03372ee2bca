"""Cameras for the benchmark views, generated on the GPU by ``vt_raygen``.

``Camera.pinhole`` reproduces the reference's ``generate_camera_rays``
(vorotracing/utils/__init__.py:85-130).  The fisheye, rolling-shutter and
thin-lens models have no counterpart in the reference; they produce the
non-pinhole view of the C5 benchmark configuration, whose rays need a start
cell each (``InferScene.render(..., per_ray_start=True)``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import check, lib, ptr, stream_ptr

PINHOLE, FISHEYE, ROLLING, THIN_LENS = 0, 1, 2, 3


class VtCamera(C.Structure):
    _fields_ = [("K", C.c_float * 4), ("c2w", C.c_float * 12), ("width", C.c_uint32),
                ("height", C.c_uint32), ("spp", C.c_uint32), ("model", C.c_int32),
                ("rs_duration", C.c_float), ("velocity", C.c_float * 3),
                ("lens_radius", C.c_float), ("focus_distance", C.c_float),
                ("seed", C.c_uint32)]


@dataclass
class Camera:
    fx: float
    fy: float
    cx: float
    cy: float
    c2w: np.ndarray  # (4,4) or (3,4), OpenCV axes
    width: int
    height: int
    model: int = PINHOLE
    spp: int = 1
    rs_duration: float = 0.0
    velocity: tuple = (0.0, 0.0, 0.0)
    lens_radius: float = 0.0
    focus_distance: float = 1.0
    seed: int = 0

    @classmethod
    def pinhole(cls, K, c2w, width, height):
        K = np.asarray(K, np.float64)
        return cls(K[0, 0], K[1, 1], K[0, 2], K[1, 2], np.asarray(c2w), width, height)

    @classmethod
    def fisheye(cls, c2w, width, height, fov_deg=190.0):
        """Equidistant fisheye whose horizontal field of view is fov_deg."""
        f = (width / 2.0) / np.radians(fov_deg / 2.0)
        return cls(f, f, width / 2.0, height / 2.0, np.asarray(c2w), width, height, FISHEYE)

    def struct(self) -> VtCamera:
        M = np.asarray(self.c2w, np.float64)[:3, :4].reshape(-1)
        return VtCamera((C.c_float * 4)(self.fx, self.fy, self.cx, self.cy),
                        (C.c_float * 12)(*M), self.width, self.height, self.spp, self.model,
                        self.rs_duration, (C.c_float * 3)(*self.velocity), self.lens_radius,
                        self.focus_distance, self.seed & 0xFFFFFFFF)

    def rays(self, device=None) -> torch.Tensor:
        """(H, W, 6) for spp == 1, else (H, W, spp, 6) float32 on the GPU."""
        dev = device or torch.device("cuda", torch.cuda.current_device())
        shape = (self.height, self.width) + ((self.spp,) if self.spp > 1 else ()) + (6,)
        out = torch.empty(shape, dtype=torch.float32, device=dev)
        st = self.struct()
        check(lib().vt_raygen(C.byref(st), ptr(out), stream_ptr(dev)), "vt_raygen")
        return out
