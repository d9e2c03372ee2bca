"""Oracle parity of the R=8 kernels the benchmark configurations run.

The reference compiles its kernels for 8x8 octahedral maps only
(vorotracing/cuda/csrc/tracing/tracing_octmap.cu:27-28), so these tests hold
the R=8 instantiations to the CPU oracle on the benchmark scenes themselves:

* the training backward (tracing_octmap.cu:232-340, ray_integrator_octmap.cuh:
  635-1027) on a strided sample of C4's rays (3M sites), fp32 and fp16
  attributes, with the upstream gradient of an MSE loss against a seeded
  target, walking and replaying the forward's path record;
* q8 inference (tracing_octmap.cu:723-779, ray_integrator_octmap.cuh:463-633)
  on a C3 view (1M sites, Morton-sorted, 4x8 tiles), bit-exact;
* the ``TraceVoroTracing`` autograd function (vorotracing/cuda/_wrapper.py:
  22-231) on an R=8 scene of C1's size, including the ``cell_distortion_gate``
  two-pass backward (_wrapper.py:145-171).

Tolerances.  fp32 gradients: relative 1e-3 (the north star's bound) plus an
absolute 1e-4 of the array's largest magnitude for elements that are the small
difference of large terms (the GPU sums with atomics in another order).
fp16 texel gradients are summed in fp32 and rounded once by the kernel, and
the oracle sums in fp32 too: they must lie within one binary16 ulp of the
oracle's sum rounded to binary16, plus the same absolute term.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import close_f16

pytestmark = pytest.mark.gpu

STRIDE = 397  # every 397th ray of a C4 frame (4,066 rays)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _close_f32(got, ref, name, rtol=1e-3, abs_frac=1e-4):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    scale = max(float(np.abs(ref).max()), 1e-30)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=abs_frac * scale, err_msg=name)


# ---------------------------------------------------------------- C4 backward at R=8

@pytest.fixture(scope="module")
def c4_sample():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cuda import NNBVH

    s = sc.config_scene("C4", adjacency="gpu", cache=False)
    W, H = sc.CONFIGS["C4"]["W"], sc.CONFIGS["C4"]["H"]
    rays = sc.pinhole_rays(sc.intrinsics(W, H), sc.orbit_pose(0, 64), W, H).reshape(-1, 6)
    rays = np.ascontiguousarray(rays[::STRIDE])
    pts = _dev(s["points"])
    bvh = NNBVH()
    bvh.build(pts)
    st = int(bvh.query(pts, _dev(rays[:1, :3]))[0])
    start = np.full(rays.shape[0], st, np.uint32)
    target = np.random.default_rng(44).uniform(0, 1, (rays.shape[0], 4)).astype(np.float32)
    return s, rays, start, target


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("replay", [False, True], ids=["walk", "replay"])
def test_c4_r8_backward_matches_oracle(c4_sample, half, replay):
    from vorotracing_b200.cuda import _ops

    s, rays, start, target = c4_sample
    assert s["res"] == 8
    nr = rays.shape[0]
    adt = np.float16 if half else np.float32
    dif, spe = s["diffuse"].astype(adt), s["specular"].astype(adt)
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dif, spe,
                     oracle.ATTR_F16 if half else oracle.ATTR_F32)
    g = dict(points=_dev(s["points"]), diffuse=_dev(dif), specular=_dev(spe),
             density=_dev(s["density"]), adj=_dev(s["adj"]), offs=_dev(s["offs"]))
    args = (g["points"], g["diffuse"], g["specular"], g["density"], g["adj"], g["offs"],
            _dev(rays), _dev(start))
    path = _ops.PathRecord(nr, 256, "cuda") if replay else None
    f = _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False, path=path)
    torch.cuda.synchronize()
    ref_f = oracle.trace_fwd(S, rays, start, wt=0.01)
    rgba = _host(f[0])
    if half:
        np.testing.assert_array_equal(f[0].cpu().numpy().view(np.uint16),
                                      ref_f["rgba"].view(np.uint16))
    else:
        np.testing.assert_array_equal(rgba, ref_f["rgba"])
    # dL/drgba of mean((rgba - target)^2), in the attributes' dtype as the op requires
    grad = (2.0 * (rgba.astype(np.float32) - target) / rgba.size).astype(adt)
    # scale up so the fp16 gradients are not subnormal
    grad = (grad.astype(np.float32) * 1024.0).astype(adt)
    res = _ops.trace_vorotracing_bwd(*args, f[0], _dev(grad), None, None, None, None, 0.0, f[5],
                                     None, f[6], f[7], f[8], 0.01, 1024, path=path)
    torch.cuda.synchronize()
    ref = oracle.trace_bwd(S, rays, start, ref_f["rgba"], grad, W=ref_f["W"], S=ref_f["S"],
                           t_far=ref_f["t_far"], distortion=ref_f["distortion"], wt=0.01)
    _close_f32(_host(res[0]), ref["points"], "points")
    _close_f32(_host(res[3]), ref["density"], "density")
    if half:
        close_f16(_host(res[1]), ref["diffuse"], "diffuse")
        close_f16(_host(res[2]), ref["specular"], "specular")
    else:
        _close_f32(_host(res[1]), ref["diffuse"], "diffuse")
        _close_f32(_host(res[2]), ref["specular"], "specular")
    # the gradients are not trivially zero
    assert np.count_nonzero(ref["diffuse"]) > 1000 and np.count_nonzero(ref["points"]) > 1000


def test_c4_r8_backward_extras_match_oracle(c4_sample):
    """Depth quantiles, distortion, ray error and the contribution term at R=8."""
    from vorotracing_b200.cuda import _ops

    s, rays, start, target = c4_sample
    nr = rays.shape[0]
    rng = np.random.default_rng(45)
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], s["diffuse"],
                     s["specular"], oracle.ATTR_F32)
    dq = np.ascontiguousarray(np.sort(rng.uniform(0.05, 0.95, (nr, 3)).astype(np.float32),
                                      axis=1)[:, ::-1])
    args = (_dev(s["points"]), _dev(s["diffuse"]), _dev(s["specular"]), _dev(s["density"]),
            _dev(s["adj"]), _dev(s["offs"]), _dev(rays), _dev(start))
    f = _ops.trace_vorotracing_fwd(*args, _dev(dq), 0.01, 1024, False)
    ref_f = oracle.trace_fwd(S, rays, start, depth_quantiles=dq, wt=0.01)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_host(f[1]).reshape(-1, 3), ref_f["depth"])
    np.testing.assert_array_equal(_host(f[5]).reshape(-1), ref_f["distortion"])
    grad = 2.0 * (ref_f["rgba"] - target) / ref_f["rgba"].size
    dgrad = rng.normal(0, 1e-3, (nr, 3)).astype(np.float32)
    err = rng.uniform(0, 1, nr).astype(np.float32)
    distg = np.full(nr, 0.01 / nr, np.float32)
    res = _ops.trace_vorotracing_bwd(*args, f[0], _dev(grad.astype(np.float32)), _dev(dq), f[2],
                                     _dev(dgrad), _dev(err), 0.25, f[5], _dev(distg), f[6],
                                     f[7], f[8], 0.01, 1024)
    torch.cuda.synchronize()
    ref = oracle.trace_bwd(S, rays, start, ref_f["rgba"], grad, depth_quantiles=dq,
                           depth_idx=ref_f["depth_idx"], depth_grad=dgrad, ray_error=err,
                           contribution_alpha_grad=0.25, distortion=ref_f["distortion"],
                           distortion_grad=distg, W=ref_f["W"], S=ref_f["S"],
                           t_far=ref_f["t_far"], wt=0.01)
    for k, name in ((0, "points"), (1, "diffuse"), (2, "specular"), (3, "density")):
        _close_f32(_host(res[k]), ref[name], name)
    _close_f32(_host(res[5]), ref["point_error"], "point_error")


# ---------------------------------------------------------------- C3 q8 inference at R=8

def test_c3_q8_r8_view_matches_oracle():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.render import InferScene

    s = sc.config_scene("C3", adjacency="gpu", cache=False)
    assert s["res"] == 8
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]), quantize="q8", sort_morton=True)
    W, H = sc.CONFIGS["C3"]["W"], sc.CONFIGS["C3"]["H"]
    rays_np = sc.pinhole_rays(sc.intrinsics(W, H), sc.orbit_pose(5, 64), W, H)
    rays = _dev(rays_np)
    rgba = scene.render(rays, weight_threshold=0.01, cell_skip_threshold=1e-3)
    torch.cuda.synchronize()
    q8 = tuple(np.float32(v) for v in (scene.diff_scale, scene.diff_offset, scene.spec_scale,
                                       scene.spec_offset))
    S = oracle.Scene(_host(scene.primal_points), _host(scene.point_adjacency),
                     _host(scene.point_adjacency_offsets), _host(scene.density),
                     _host(scene.diffuse_q8), _host(scene.specular_q8), oracle.ATTR_U8, q8=q8)
    start = _host(scene.get_starting_point(rays)).reshape(-1)
    idx = np.arange(0, H * W, 131)
    ref = oracle.trace_infer(S, rays_np.reshape(-1, 6)[idx], start[idx], wt=0.01, skip=1e-3)
    got = rgba.reshape(-1, 4).cpu().numpy()[idx]
    np.testing.assert_array_equal(got.view(np.uint16), ref["rgba"].view(np.uint16))
    assert float(np.asarray(ref["rgba"][:, 3], np.float32).mean()) > 0.1


# ---------------------------------------------------------------- TraceVoroTracing vs oracle

@pytest.fixture(scope="module")
def r8_small():
    from vorotracing_b200 import scene as sc

    s = sc.make_scene(16384, 7, False, 8)
    rays = sc.pinhole_rays(sc.intrinsics(64, 48), sc.look_at((0.0, 0.4, 2.9), up=(0, 1, 0)),
                           64, 48)
    st = oracle.nn_query(s["points"], rays.reshape(-1, 6)[:1, :3])[0]
    return s, rays, np.full(64 * 48, st, np.uint32)


@pytest.mark.parametrize("gate", [False, True], ids=["plain", "distortion_gate"])
def test_autograd_function_matches_oracle(r8_small, gate):
    from vorotracing_b200.cuda import TraceVoroTracing

    s, rays_np, start_np = r8_small
    H, W = rays_np.shape[:2]
    nr = H * W
    rng = np.random.default_rng(46)
    dq = np.ascontiguousarray(np.sort(rng.uniform(0.1, 0.9, (nr, 2)).astype(np.float32),
                                      axis=1)[:, ::-1])
    target = rng.uniform(0, 1, (H, W, 4)).astype(np.float32)
    err = rng.uniform(0, 1, (H, W)).astype(np.float32)
    cgate = rng.uniform(0, 2, (s["points"].shape[0], 1)).astype(np.float32)
    lam_d, lam_z, lam_c = 0.05, 1e-3, 0.5
    params = [_dev(s[k]).requires_grad_() for k in ("points", "diffuse", "specular", "density")]
    rgba, depth, contrib, n_int, errbox, dist = TraceVoroTracing.apply(
        *params, _dev(s["adj"]), _dev(s["offs"]), _dev(rays_np), _dev(start_np).view(H, W),
        _dev(dq).view(H, W, 2), 0.01, 1024, True)
    errbox.ray_error = _dev(err)
    if gate:
        errbox.cell_distortion_gate = _dev(cgate)
    loss = (((rgba - _dev(target)) ** 2).mean() + lam_d * dist.mean() + lam_z * depth.sum()
            + lam_c * contrib.sum())
    loss.backward()
    torch.cuda.synchronize()

    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], s["diffuse"], s["specular"],
                     oracle.ATTR_F32)
    rays = rays_np.reshape(-1, 6)
    f = oracle.trace_fwd(S, rays, start_np, depth_quantiles=dq, wt=0.01)
    np.testing.assert_array_equal(_host(rgba).reshape(-1, 4), f["rgba"])
    g_rgba = (2.0 * (f["rgba"] - target.reshape(-1, 4)) / f["rgba"].size).astype(np.float32)
    g_dist = np.full(nr, lam_d / nr, np.float32)
    g_depth = np.full((nr, 2), lam_z, np.float32)
    common = dict(depth_quantiles=dq, depth_idx=f["depth_idx"], W=f["W"], S=f["S"],
                  t_far=f["t_far"], distortion=f["distortion"], wt=0.01)
    if gate:
        # _wrapper.py:145-171: density gets main + gate * distortion-only; the
        # other gradients come from the main pass alone
        dpass = oracle.trace_bwd(S, rays, start_np, f["rgba"], np.zeros_like(g_rgba),
                                 depth_grad=np.zeros_like(g_depth), distortion_grad=g_dist,
                                 **common)
        ref = oracle.trace_bwd(S, rays, start_np, f["rgba"], g_rgba, depth_grad=g_depth,
                               ray_error=err.reshape(-1), contribution_alpha_grad=lam_c,
                               distortion_grad=np.zeros_like(g_dist), **common)
        ref["density"] = ref["density"] + cgate.reshape(-1) * dpass["density"]
    else:
        ref = oracle.trace_bwd(S, rays, start_np, f["rgba"], g_rgba, depth_grad=g_depth,
                               ray_error=err.reshape(-1), contribution_alpha_grad=lam_c,
                               distortion_grad=g_dist, **common)
    for p, name in zip(params, ("points", "diffuse", "specular", "density")):
        _close_f32(_host(p.grad), np.nan_to_num(ref[name]), name)
    _close_f32(_host(errbox.point_error), ref["point_error"], "point_error")
