import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


from oracle import pad_f16x4, quantize_u8  # noqa: E402,F401  (re-exported for the tests)


@pytest.fixture(scope="session")
def c1_scene():
    from vorotracing_b200 import scene as sc

    return sc.config_scene("C1")


@pytest.fixture(scope="session")
def c1_rays():
    from vorotracing_b200 import scene as sc

    return sc.config_rays("C1")


def tile_perm(H: int, W: int, TH: int = 4, TW: int = 8) -> np.ndarray:
    """The reference's _tile_perm key (vorotracing.py:606-625), stable argsort."""
    y, x = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    tpr = (W + TW - 1) // TW
    k = ((y // TH) * tpr + (x // TW)) * (TH * TW) + (y % TH) * TW + (x % TW)
    return np.argsort(k.reshape(-1), kind="stable").astype(np.int32)
