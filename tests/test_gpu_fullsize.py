"""Parity at the benchmark configurations' full sizes.

The whole frame / batch runs on the GPU; the CPU oracle checks a strided
sample of its rays bit for bit, and size-independent properties cover the
rest: the 4x8 tile order and the host-memory render leave every pixel
unchanged, per-ray start cells equal the broadcast one for a pinhole camera,
and the backward's path-record replay gives the gradients of a full walk.
Scenes use the GPU Voronoi adjacency (the Qhull build takes minutes at these
sizes).
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

SAMPLE = 257  # every 257th ray is checked against the oracle


def _host(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def c2():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.render import InferScene

    s = sc.config_scene("C2", adjacency="gpu", cache=False)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    scene = InferScene(d(s["points"]), d(s["density"]), d(s["adj"]), d(s["offs"]),
                       d(s["diffuse"]), d(s["specular"]), quantize="fp16", sort_morton=True)
    rays = sc.config_rays("C2")
    return scene, rays


def test_c2_full_frame_matches_oracle(c2):
    scene, rays_np = c2
    H, W = rays_np.shape[:2]
    rays = torch.from_numpy(rays_np).cuda()
    rgba = scene.render(rays, weight_threshold=0.01, cell_skip_threshold=1e-3)
    torch.cuda.synchronize()
    assert rgba.shape == (H, W, 4)
    S = oracle.Scene(_host(scene.primal_points), _host(scene.point_adjacency),
                     _host(scene.point_adjacency_offsets), _host(scene.density),
                     _host(scene.diffuse_fp16), _host(scene.specular_fp16), oracle.ATTR_F16X4)
    start = _host(scene.get_starting_point(rays)).reshape(-1)
    idx = np.arange(0, H * W, SAMPLE)
    ref = oracle.trace_infer(S, rays_np.reshape(-1, 6)[idx], start[idx], wt=0.01, skip=1e-3)
    got = _host(rgba).reshape(-1, 4)[idx]
    np.testing.assert_array_equal(got.view(np.uint16), ref["rgba"].view(np.uint16))


def test_c2_full_frame_invariances(c2):
    """Tile order, per-ray start cells and host-memory I/O change no pixel."""
    scene, rays_np = c2
    rays = torch.from_numpy(rays_np).cuda()
    kw = dict(weight_threshold=0.01, cell_skip_threshold=1e-3)
    a = scene.render(rays, **kw)
    b = scene.render(rays, use_warp_perm=False, **kw)
    c = scene.render(rays, per_ray_start=True, **kw)
    host = torch.from_numpy(rays_np).pin_memory()
    e = scene.render_host(host, **kw)
    f = scene.render_host(host, transfer="bands", bands=5, **kw)
    torch.cuda.synchronize()
    ref = a.view(torch.int16)
    for other in (b, c):
        assert torch.equal(other.view(torch.int16), ref)
    for other in (e, f):
        assert torch.equal(other.view(torch.int16), ref.cpu())


@pytest.fixture(scope="module")
def c4():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cuda import NNBVH, _ops

    s = sc.config_scene("C4", adjacency="gpu", cache=False)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    t = {k: d(s[k]) for k in ("points", "density", "diffuse", "specular", "adj", "offs")}
    W, H = sc.CONFIGS["C4"]["W"], sc.CONFIGS["C4"]["H"]
    rays = d(sc.pinhole_rays(sc.intrinsics(W, H), sc.orbit_pose(0, 64), W, H))
    bvh = NNBVH()
    bvh.build(t["points"])
    st = bvh.query(t["points"], rays[0, 0, :3].reshape(1, 3))
    start = st.expand(H * W).contiguous().view(torch.uint32)
    perm = _ops.tile_perm(H, W, device="cuda").long()
    rays = rays.reshape(-1, 6)[perm].contiguous()
    return s, t, rays, start


def test_c4_full_batch_forward_matches_oracle(c4):
    from vorotracing_b200.cuda import _ops

    s, t, rays, start = c4
    nr = rays.size(0)
    path = _ops.PathRecord(nr, 256, "cuda")
    out = _ops.trace_vorotracing_fwd(t["points"], t["diffuse"], t["specular"], t["density"],
                                     t["adj"], t["offs"], rays, start, None, 0.01, 1024, False,
                                     path=path)
    torch.cuda.synchronize()
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], s["diffuse"], s["specular"],
                     oracle.ATTR_F32)
    idx = np.arange(0, nr, SAMPLE)
    r = _host(rays)[idx]
    ref = oracle.trace_fwd(S, r, _host(start)[idx], wt=0.01)
    np.testing.assert_array_equal(_host(out[0])[idx], ref["rgba"])
    np.testing.assert_array_equal(_host(out[4]).reshape(-1)[idx], ref["n"])
    for k, name in ((5, "distortion"), (6, "W"), (7, "S"), (8, "t_far")):
        np.testing.assert_array_equal(_host(out[k]).reshape(-1)[idx], ref[name], err_msg=name)


def test_c4_full_batch_replay_equals_walk(c4):
    """The backward replaying the forward's record (cells and colours)
    returns the gradients of the backward that walks every ray."""
    from vorotracing_b200.cuda import _ops

    s, t, rays, start = c4
    nr = rays.size(0)
    args = (t["points"], t["diffuse"], t["specular"], t["density"], t["adj"], t["offs"], rays,
            start)
    path = _ops.PathRecord(nr, 256, "cuda")
    f = _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False, path=path)
    g = torch.randn(f[0].shape, generator=torch.Generator("cuda").manual_seed(3),
                    device="cuda") * 1e-6
    common = (f[0], g, None, None, None, None, 0.0, f[5], None, f[6], f[7], f[8], 0.01, 1024)
    walk = _ops.trace_vorotracing_bwd(*args, *common)
    rep = _ops.trace_vorotracing_bwd(*args, *common, path=path)
    flagged = int(((path.len.view(torch.int32) < 0)).sum())
    assert flagged < nr // 10
    for a, b, name in zip(walk[:4], rep[:4], ("points", "diffuse", "specular", "density")):
        scale = float(a.abs().max())
        torch.testing.assert_close(b, a, rtol=1e-3, atol=1e-4 * scale, msg=name)


def test_c5_full_start_cells():
    """Per-ray start cells of non-pinhole cameras (4M sites): the hinted BVH
    search equals the unhinted one everywhere and the brute-force nearest
    site on a sample."""
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cameras import ROLLING, THIN_LENS, Camera
    from vorotracing_b200.cuda import NNBVH

    s = sc.config_scene("C5", adjacency="gpu", cache=False)
    pts = torch.from_numpy(s["points"]).cuda()
    bvh = NNBVH()
    bvh.build(pts)
    W, H = sc.CONFIGS["C5"]["W"], sc.CONFIGS["C5"]["H"]
    K, T = sc.intrinsics(W, H), sc.orbit_pose(0, 64)
    rs = Camera.pinhole(K, T, W, H)
    rs.model, rs.rs_duration, rs.velocity = ROLLING, 0.03, tuple(T[:3, 0])
    tl = Camera.pinhole(K, T, W, H)
    tl.model, tl.spp, tl.lens_radius, tl.focus_distance, tl.seed = THIN_LENS, 4, 0.02, 3.0, 5
    for cam in (rs, tl):
        o = cam.rays("cuda").reshape(-1, 6)[:, :3].contiguous()
        plain = bvh.query(pts, o)
        hinted = bvh.query(pts, o, hint=plain[:1])
        assert torch.equal(plain, hinted)
        idx = np.arange(0, o.size(0), o.size(0) // 64)
        np.testing.assert_array_equal(_host(plain)[idx], oracle.nn_query(s["points"], _host(o)[idx]))
