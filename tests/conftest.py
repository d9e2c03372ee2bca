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


def close_f16(got, ref32, name="", abs_frac=1e-4):
    """A binary16 result against an fp32 sum: within one binary16 ulp of the
    sum rounded to binary16, plus abs_frac of the array's largest magnitude
    (elements that are the small difference of large terms carry the fp32
    rounding of a different summation order)."""
    got = np.asarray(got, np.float64).reshape(-1)
    ref16 = np.asarray(ref32, np.float32).reshape(-1).astype(np.float16)
    ulp = np.maximum(np.spacing(np.abs(ref16)).astype(np.float64), 2.0 ** -24)
    scale = max(float(np.abs(np.asarray(ref32, np.float64)).max()), 1e-30)
    err = np.abs(got - ref16.astype(np.float64))
    bad = np.flatnonzero(err > ulp + abs_frac * scale)
    assert bad.size == 0, (f"{name}: {bad.size} of {got.size} elements beyond 1 binary16 ulp; "
                           f"first {bad[:5]} got {got[bad[:5]]} want {ref16[bad[:5]]}")
