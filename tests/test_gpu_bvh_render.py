"""Start-cell BVH against the oracle's brute-force nearest site, and the
end-to-end InferScene render (Morton reorder + BVH + tile order + trace)
against the oracle on the original cell order."""
import numpy as np
import pytest
import torch

import oracle
from tests.conftest import pad_f16x4, quantize_u8

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_bvh_matches_brute_force(c1_scene):
    from vorotracing_b200.cuda import NNBVH

    pts = c1_scene["points"]
    rng = np.random.default_rng(7)
    q = np.concatenate([rng.uniform(-3, 3, (20000, 3)), pts[:500], pts[:500] + 1e-4,
                        rng.uniform(-50, 50, (100, 3))]).astype(np.float32)
    b = NNBVH()
    b.build(_dev(pts))
    got = b.query(_dev(pts), _dev(q)).cpu().numpy()
    ref = oracle.nn_query(pts, q)
    np.testing.assert_array_equal(got, ref)
    # a hint (good, bad, or one per query) never changes the answer
    for hint in (torch.tensor([int(ref[0])]), torch.tensor([12345]),
                 torch.from_numpy(rng.integers(0, len(pts), len(q)).astype(np.int32))):
        got = b.query(_dev(pts), _dev(q), hint=hint.cuda()).cpu().numpy()
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("spread", [0.0, 1e-3, 2e-2, 0.3])
def test_bvh_warp_cooperative_queries(c1_scene, spread):
    """Warps of 32 close queries (ray origins of a tile, a lens aperture) take
    the warp-cooperative traversal, scattered ones the per-lane search; either
    way every answer is the brute-force (d2, lowest id) minimum, with and
    without hints.  Spread 0 puts 32 identical queries in a warp, and some
    clusters sit exactly between sites (ties)."""
    from vorotracing_b200.cuda import NNBVH

    pts = c1_scene["points"]
    rng = np.random.default_rng(11)
    centres = np.concatenate([rng.uniform(-2.5, 2.5, (60, 3)),
                              0.5 * (pts[:4] + pts[4:8])]).astype(np.float32)
    q = (np.repeat(centres, 32, axis=0)
         + spread * rng.standard_normal((len(centres) * 32, 3))).astype(np.float32)
    q = np.concatenate([q, rng.uniform(-3, 3, (17, 3)).astype(np.float32)])  # ragged last warp
    b = NNBVH()
    b.build(_dev(pts))
    ref = oracle.nn_query(pts, q)
    np.testing.assert_array_equal(b.query(_dev(pts), _dev(q)).cpu().numpy(), ref)
    for hint in (torch.tensor([int(ref[0])]), torch.tensor([len(pts) - 1]),
                 torch.from_numpy(np.roll(ref, 1).astype(np.int32))):
        got = b.query(_dev(pts), _dev(q), hint=hint.cuda()).cpu().numpy()
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("n", [1, 2, 3, 33])
def test_bvh_tiny_and_duplicates(n):
    from vorotracing_b200.cuda import nearest_neighbor_bvh

    rng = np.random.default_rng(n)
    pts = rng.integers(0, 2, (n, 3)).astype(np.float32)  # duplicates for n > 8
    q = rng.uniform(-1, 2, (257, 3)).astype(np.float32)
    got = nearest_neighbor_bvh(_dev(pts), _dev(q)).cpu().numpy()
    ref = oracle.nn_query(pts, q)
    np.testing.assert_array_equal(got, ref)
    from vorotracing_b200.cuda import NNBVH

    b = NNBVH()
    b.build(_dev(pts))
    hint = torch.tensor([n - 1], dtype=torch.int32).cuda()  # ties must still go to the lowest id
    np.testing.assert_array_equal(b.query(_dev(pts), _dev(q), hint=hint).cpu().numpy(), ref)


@pytest.mark.parametrize("quant", ["fp16", "q8"])
def test_infer_scene_matches_oracle(c1_scene, c1_rays, quant):
    from vorotracing_b200.render import InferScene

    s = c1_scene
    res = s["res"]
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]), quantize=quant, sort_morton=True)
    rgba = scene.render(_dev(c1_rays), weight_threshold=0.01, cell_skip_threshold=1e-3)
    torch.cuda.synchronize()
    start = oracle.nn_query(s["points"], c1_rays.reshape(-1, 6)[:1, :3])
    start = np.full(c1_rays.shape[0] * c1_rays.shape[1], start[0], np.uint32)
    if quant == "fp16":
        S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"],
                         pad_f16x4(s["diffuse"], res), pad_f16x4(s["specular"], res),
                         oracle.ATTR_F16X4)
    else:
        dq, ds, do = quantize_u8(s["diffuse"])
        sq, ss, so = quantize_u8(s["specular"])
        S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dq, sq, oracle.ATTR_U8,
                         q8=(ds, do, ss, so))
    ref = oracle.trace_infer(S, c1_rays, start, wt=0.01, skip=1e-3)
    np.testing.assert_array_equal(rgba.reshape(-1, 4).cpu().numpy().view(np.uint16),
                                  ref["rgba"].view(np.uint16))


@pytest.mark.parametrize("transfer,bands", [("zero_copy", 1), ("bands", 1), ("bands", 3),
                                            ("bands", 4), ("bands", 7)])
def test_render_host_roundtrip(c1_scene, c1_rays, transfer, bands):
    from vorotracing_b200.render import InferScene

    s = c1_scene
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]))
    host = torch.from_numpy(c1_rays).pin_memory()
    out = scene.render_host(host, transfer=transfer, bands=bands, weight_threshold=0.01)
    dev = scene.render(_dev(c1_rays), weight_threshold=0.01).cpu()
    assert torch.equal(out.view(torch.int16), dev.view(torch.int16))
    # unpinned host buffers work too (staged through page-locked ones)
    plain = scene.render_host(torch.from_numpy(c1_rays.copy()), torch.empty_like(out),
                              transfer=transfer, bands=bands, weight_threshold=0.01)
    assert torch.equal(plain.view(torch.int16), dev.view(torch.int16))
    # a second call reuses the device ray buffer; odd row counts leave a short last band
    out2 = scene.render_host(host[:-5].clone().pin_memory(), transfer=transfer, bands=bands, weight_threshold=0.01)
    assert torch.equal(out2.view(torch.int16), dev[:-5].view(torch.int16))


def test_render_host_async_unpinned_rays(c1_scene, c1_rays):
    """sync=False with unpinned rays: the staged page-locked copy stays alive
    while the trace reads it, even when other page-locked buffers are
    allocated and scribbled on before the trace finishes."""
    from vorotracing_b200.render import InferScene

    s = c1_scene
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]))
    want = scene.render(_dev(c1_rays), weight_threshold=0.01).cpu()
    outs = []
    for _ in range(4):
        outs.append(scene.render_host(torch.from_numpy(c1_rays.copy()), sync=False,
                                      weight_threshold=0.01))
        junk = torch.empty(c1_rays.shape, dtype=torch.float32, pin_memory=True)
        junk.fill_(float("nan"))
        del junk
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("mode", ["mean", "quantile"])
def test_render_depth_matches_oracle(c1_scene, c1_rays, mode):
    """Fused depth render vs the oracle's training forward with the same
    thresholds for every ray, averaged as the reference viewer does."""
    from vorotracing_b200.render import InferScene

    s = c1_scene
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]))
    n = 6
    thr = (np.linspace(1 - 1 / (2 * n), 1 / (2 * n), n) if mode == "mean"
           else np.array([0.3])).astype(np.float32)
    depth = scene.render_depth(_dev(c1_rays), mode=mode, thresholds=_dev(thr),
                               weight_threshold=0.001).cpu().numpy().reshape(-1)
    nr = c1_rays.shape[0] * c1_rays.shape[1]
    start = oracle.nn_query(s["points"], c1_rays.reshape(-1, 6)[:1, :3])
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], s["diffuse"], s["specular"],
                     oracle.ATTR_F32)
    f = oracle.trace_fwd(S, c1_rays, np.full(nr, start[0], np.uint32),
                         depth_quantiles=np.tile(thr, (nr, 1)), wt=0.001)
    d = f["depth"]
    if mode == "mean":
        ref = np.full(nr, -1.0, np.float32)
        for r in range(nr):
            v = [x for x in d[r] if x > 0]
            if v:
                acc = np.float32(0)
                for x in v:
                    acc = np.float32(acc + np.float32(x))
                ref[r] = acc / np.float32(len(v))
    else:
        ref = d[:, 0]
    np.testing.assert_array_equal(depth, ref)
