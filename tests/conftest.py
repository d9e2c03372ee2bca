import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def c1_scene():
    from vorotracing_b200 import scene as sc

    return sc.config_scene("C1")


@pytest.fixture(scope="session")
def c1_rays():
    from vorotracing_b200 import scene as sc

    return sc.config_rays("C1")


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


def tile_perm(H: int, W: int, TH: int = 4, TW: int = 8) -> np.ndarray:
    """The reference's _tile_perm key (vorotracing.py:606-625), stable argsort."""
    y, x = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    tpr = (W + TW - 1) // TW
    k = ((y // TH) * tpr + (x // TW)) * (TH * TW) + (y % TH) * TW + (x % TW)
    return np.argsort(k.reshape(-1), kind="stable").astype(np.int32)
