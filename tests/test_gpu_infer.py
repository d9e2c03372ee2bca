"""Parity of the fp16 / q8 inference kernels against the CPU oracle.

Bit-exact: visited-cell sequences, per-ray step / face / segment / texture
counters and the binary16 rgba words (the kernels and the oracle evaluate the
same IEEE binary32 operation sequence).
"""
import numpy as np
import pytest
import torch

import oracle
from tests.conftest import pad_f16x4, quantize_u8, tile_perm

pytestmark = pytest.mark.gpu

SEQ_CAP = 256


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gpu_scene(s):
    from vorotracing_b200 import cuda as ops

    pts = _dev(s["points"])
    adj = _dev(s["adj"])
    offs = _dev(s["offs"])
    den = _dev(s["density"])
    faces = ops.prefetch_octmap_adj(pts, adj, offs)
    return pts, adj, offs, den, faces


def _start(s, rays):
    st = oracle.nn_query(s["points"], rays.reshape(-1, 6)[:1, :3])
    return np.full(rays.reshape(-1, 6).shape[0], st[0], np.uint32)


def _u32(a):
    return _dev(np.asarray(a, np.uint32))


@pytest.mark.parametrize("perm", [False, True])
@pytest.mark.parametrize("skip", [0.0, 1e-3])
def test_infer_f16_bit_exact(c1_scene, c1_rays, perm, skip):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    res = s["res"]
    dif = pad_f16x4(s["diffuse"], res)
    spe = pad_f16x4(s["specular"], res)
    start = _start(s, c1_rays)
    ref = oracle.trace_infer(oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dif, spe,
                                          oracle.ATTR_F16X4), c1_rays, start, wt=0.01, skip=skip,
                             seq_cap=SEQ_CAP)
    pts, adj, offs, den, faces = _gpu_scene(s)
    H, W = c1_rays.shape[:2]
    rp = _dev(tile_perm(H, W)) if perm else torch.empty(0, dtype=torch.int32, device="cuda")
    dbg = {"seq_cap": SEQ_CAP}
    rgba = _ops.trace_vorotracing_infer(pts, _dev(dif), _dev(spe), den, adj, offs, _dev(c1_rays),
                                        _u32(start).view(H, W), faces, rp, 0.01, 1024, skip,
                                        debug=dbg)
    torch.cuda.synchronize()
    assert rgba.shape == (H, W, 4) and rgba.dtype == torch.float16
    np.testing.assert_array_equal(dbg["seq_len"].cpu().numpy(), ref["seq_len"].astype(np.int32))
    np.testing.assert_array_equal(dbg["seq"].cpu().numpy(), ref["seq"].astype(np.int32))
    np.testing.assert_array_equal(dbg["stats"].cpu().numpy(), ref["stats"].astype(np.int32))
    got = rgba.reshape(-1, 4).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, ref["rgba"].view(np.uint16))


def test_infer_q8_bit_exact(c1_scene, c1_rays):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    dq, ds, do = quantize_u8(s["diffuse"])
    sq, ss, so = quantize_u8(s["specular"])
    start = _start(s, c1_rays)
    q8 = (np.float32(ds), np.float32(do), np.float32(ss), np.float32(so))
    ref = oracle.trace_infer(oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dq, sq,
                                          oracle.ATTR_U8, q8=q8), c1_rays, start, wt=0.01,
                             skip=1e-3, seq_cap=SEQ_CAP)
    pts, adj, offs, den, faces = _gpu_scene(s)
    dbg = {"seq_cap": SEQ_CAP}
    rgba = _ops.trace_vorotracing_infer_q8(pts, _dev(dq), _dev(sq), den, adj, offs, _dev(c1_rays),
                                           _u32(start), faces, ds, do, ss, so, 0.01, 1024, 1e-3,
                                           debug=dbg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dbg["seq"].cpu().numpy(), ref["seq"].astype(np.int32))
    got = rgba.reshape(-1, 4).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, ref["rgba"].view(np.uint16))


@pytest.mark.parametrize("max_int", [1, 3, 17])
def test_infer_max_intersections(c1_scene, c1_rays, max_int):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    res = s["res"]
    dif, spe = pad_f16x4(s["diffuse"], res), pad_f16x4(s["specular"], res)
    rays = c1_rays[::7, ::5]
    start = _start(s, rays)
    ref = oracle.trace_infer(oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dif, spe,
                                          oracle.ATTR_F16X4), rays, start, wt=0.0,
                             max_int=max_int)
    pts, adj, offs, den, faces = _gpu_scene(s)
    dbg = {}
    rgba = _ops.trace_vorotracing_infer(pts, _dev(dif), _dev(spe), den, adj, offs,
                                        _dev(rays), _u32(start), faces, None, 0.0, max_int, 0.0,
                                        debug=dbg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dbg["num_intersections"].cpu().numpy(), ref["n"].astype(np.int32))
    np.testing.assert_array_equal(rgba.reshape(-1, 4).cpu().numpy().view(np.uint16),
                                  ref["rgba"].view(np.uint16))


def test_infer_empty_and_errors(c1_scene, c1_rays):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    res = s["res"]
    dif, spe = _dev(pad_f16x4(s["diffuse"], res)), _dev(pad_f16x4(s["specular"], res))
    pts, adj, offs, den, faces = _gpu_scene(s)
    empty = torch.empty(0, 6, device="cuda")
    out = _ops.trace_vorotracing_infer(pts, dif, spe, den, adj, offs, empty,
                                       torch.empty(0, dtype=torch.uint32, device="cuda"), faces,
                                       None, 0.01, 1024, 0.0)
    assert out.shape == (0, 4)
    bad = _u32(np.full(4, 10**9, np.uint32))
    with pytest.raises(RuntimeError, match="out of range"):
        _ops.trace_vorotracing_infer(pts, dif, spe, den, adj, offs, _dev(c1_rays[0, :4]), bad,
                                     faces, None, 0.01, 1024, 0.0, debug={})
    with pytest.raises(RuntimeError, match="requires float16 diffuse"):
        _ops.trace_vorotracing_infer(pts, dif.float(), spe, den, adj, offs, _dev(c1_rays[0, :4]),
                                     _u32(np.zeros(4)), faces, None, 0.01, 1024, 0.0)
    with pytest.raises(RuntimeError, match="num_points \\+ 1"):
        _ops.trace_vorotracing_infer(pts, dif, spe, den, adj, offs[:-1], _dev(c1_rays[0, :4]),
                                     _u32(np.zeros(4)), faces, None, 0.01, 1024, 0.0)


def test_prefetch_rejects_bad_csr(c1_scene):
    from vorotracing_b200 import cuda as ops

    s = c1_scene
    pts, adj, offs, den, faces = _gpu_scene(s)
    bad = adj.clone()
    bad[5] = 10**9
    with pytest.raises(RuntimeError, match="invalid Voronoi adjacency"):
        ops.prefetch_octmap_adj(pts, bad, offs)


def test_single_cell_scene():
    from vorotracing_b200.cuda import _ops
    from vorotracing_b200 import cuda as ops

    pts = torch.zeros(1, 3, device="cuda")
    adj = torch.zeros(32, dtype=torch.int32, device="cuda").view(torch.uint32)
    offs = torch.zeros(2, dtype=torch.int32, device="cuda").view(torch.uint32)
    faces = ops.prefetch_octmap_adj(pts, adj, offs)
    tex = torch.zeros(1, 4 * 64, dtype=torch.float16, device="cuda")
    rays = torch.tensor([[0.0, 0, 0, 1, 0, 0]], device="cuda")
    out = _ops.trace_vorotracing_infer(pts, tex, tex, torch.ones(1, 1, device="cuda"), adj, offs,
                                       rays, torch.zeros(1, dtype=torch.int32,
                                                         device="cuda").view(torch.uint32),
                                       faces, None, 0.01, 1024, 0.0)
    assert out.float().abs().sum().item() == 0.0


def test_infer_q8_widened_texels_identical(c1_scene, c1_rays):
    """The q8 trace on texels widened to 4 bytes (pad_u8x4, the layout
    InferScene renders from) gives the same pixels, bit for bit, as on the
    reference's 3-byte layout."""
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    dq, ds, do = quantize_u8(s["diffuse"])
    sq, ss, so = quantize_u8(s["specular"])
    wide = _ops.pad_u8x4(_dev(dq))
    w = wide.cpu().numpy().reshape(dq.shape[0], -1, 4)
    np.testing.assert_array_equal(w[..., :3].reshape(dq.shape), dq)
    assert not w[..., 3].any()
    start = _u32(_start(s, c1_rays))
    pts, adj, offs, den, faces = _gpu_scene(s)
    args = (den, adj, offs, _dev(c1_rays), start, faces, ds, do, ss, so, 0.01, 1024, 1e-3)
    a = _ops.trace_vorotracing_infer_q8(pts, _dev(dq), _dev(sq), *args)
    b = _ops.trace_vorotracing_infer_q8(pts, wide, _ops.pad_u8x4(_dev(sq)), *args)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert float(a[..., 3].float().mean()) > 0.1
