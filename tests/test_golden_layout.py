"""Layout transforms and cameras against golden vectors produced by the
reference's own Python code (tests/golden/make_golden.py).

CPU tests pin the numpy helpers the other tests use as references; GPU tests
check the CUDA layout kernels bit for bit against the same vectors."""
import os

import numpy as np
import pytest

from tests.conftest import pad_f16x4, quantize_u8, tile_perm

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "layout_golden.npz"))
TILES = [(8, 16), (13, 21), (37, 45), (5, 3)]


def morton_numpy(pts):
    pts = pts.astype(np.float32)
    lo, hi = pts.min(0), pts.max(0)
    size = np.maximum(hi - lo, np.float32(1e-6))
    norm = np.clip((pts - lo) / size * np.float32(1023.0), 0, 1023).astype(np.int64)
    code = np.zeros(len(pts), np.int64)
    for i in range(10):
        for a in range(3):
            code |= ((norm[:, a] >> i) & 1) << (3 * i + a)
    return code


@pytest.mark.parametrize("hw", TILES)
def test_tile_perm_helper(hw):
    np.testing.assert_array_equal(tile_perm(*hw), G[f"tile_{hw[0]}x{hw[1]}"])


def test_quantize_helper():
    q, s, o = quantize_u8(G["quant_src"])
    np.testing.assert_array_equal(q, G["quant_q"])
    np.testing.assert_allclose([s, o], G["quant_scale_offset"], rtol=0, atol=0)


def test_pad_helper():
    out = pad_f16x4(G["pad_src"], 8).view(np.int16)
    np.testing.assert_array_equal(out, G["pad_out"])


def test_morton_helper():
    np.testing.assert_array_equal(morton_numpy(G["morton_points"]), G["morton_codes"])


def test_camera_convention():
    from vorotracing_b200.scene import pinhole_rays

    r = pinhole_rays(G["cam_K"], G["cam_T"], 32, 24).reshape(-1, 6)
    np.testing.assert_allclose(r, G["cam_rays"], atol=2e-7, rtol=0)


# ---------------------------------------------------------------- GPU kernels

def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("hw", TILES + [(840, 1296), (1, 1), (4, 8)])
def test_tile_perm_kernel(hw):
    from vorotracing_b200.cuda import _ops

    got = _ops.tile_perm(*hw).cpu().numpy()
    ref = G[f"tile_{hw[0]}x{hw[1]}"] if hw in TILES else tile_perm(*hw)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.gpu
def test_quantize_and_pad_kernels():
    from vorotracing_b200.cuda import _ops

    q, s, o = _ops.quantize_u8(_dev(G["quant_src"]))
    np.testing.assert_array_equal(q.cpu().numpy(), G["quant_q"])
    assert (s, o) == tuple(G["quant_scale_offset"])
    p = _ops.pad_f16x4(_dev(G["pad_src"]))
    np.testing.assert_array_equal(p.cpu().numpy().view(np.int16), G["pad_out"])


@pytest.mark.gpu
def test_morton_reorder_kernels():
    import torch
    from vorotracing_b200.cuda import _ops

    pts = _dev(G["morton_points"])
    np.testing.assert_array_equal(_ops.morton_codes(pts).cpu().numpy(), G["morton_codes"])
    perm, inv = _ops.morton_perm(pts)
    np.testing.assert_array_equal(perm.cpu().numpy(), np.argsort(G["morton_codes"], kind="stable"))
    np.testing.assert_array_equal(_ops.gather_rows(pts, perm).cpu().numpy(),
                                  G["morton_new_points"])
    adj, offs = _ops.permute_csr(_dev(G["morton_adj"]), _dev(G["morton_offs"]), perm, inv)
    np.testing.assert_array_equal(offs.cpu().numpy(), G["morton_new_offs"])
    e = int(G["morton_new_offs"][-1])
    np.testing.assert_array_equal(adj.cpu().numpy()[:e], G["morton_new_adj"][:e])
    assert adj.dtype == torch.uint32


@pytest.mark.gpu
def test_morton_perm_is_stable_with_ties():
    from vorotracing_b200.cuda import _ops

    rng = np.random.default_rng(5)
    pts = rng.integers(0, 4, (5000, 3)).astype(np.float32)  # many duplicate codes
    perm, inv = _ops.morton_perm(_dev(pts))
    np.testing.assert_array_equal(perm.cpu().numpy(), np.argsort(morton_numpy(pts), kind="stable"))
    np.testing.assert_array_equal(inv.cpu().numpy()[perm.cpu().numpy()], np.arange(5000))
