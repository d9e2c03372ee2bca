"""Training forward / backward kernels against the CPU oracle.

Forward (fp32 attributes): visited-cell sequences, step counts, rgba, depth
quantiles, distortion accumulators are bit-exact; the atomically accumulated
per-cell contribution is compared with a tolerance.  Backward: every gradient
within relative 1e-3 (the gradients are atomic sums whose order differs)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import close_f16

pytestmark = pytest.mark.gpu

SEQ = 256


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _setup(s, rays, half):
    st = oracle.nn_query(s["points"], rays.reshape(-1, 6)[:1, :3])[0]
    start = np.full(rays.reshape(-1, 6).shape[0], st, np.uint32)
    dif, spe = s["diffuse"], s["specular"]
    if half:
        dif, spe = dif.astype(np.float16), spe.astype(np.float16)
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"], dif, spe,
                     oracle.ATTR_F16 if half else oracle.ATTR_F32)
    g = dict(points=_dev(s["points"]), diffuse=_dev(dif), specular=_dev(spe),
             density=_dev(s["density"]), adj=_dev(s["adj"]), offs=_dev(s["offs"]))
    return S, start, g


def _quantiles(nr, rng):
    q = np.sort(rng.uniform(0.05, 0.95, (nr, 3)).astype(np.float32), axis=1)[:, ::-1]
    return np.ascontiguousarray(q)


def _close(got, ref, rtol=1e-3, abs_frac=1e-4, name=""):
    """|got - ref| <= rtol |ref| + abs_frac max|ref|: gradients are atomic sums
    whose order differs between the GPU and the oracle, so elements that are
    the small difference of large terms carry an absolute rounding error
    proportional to the array's scale."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-12)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=abs_frac * scale, err_msg=name)


@pytest.mark.parametrize("half", [False, True])
def test_fwd_matches_oracle(c1_scene, c1_rays, half):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    rays = c1_rays[::2, ::2]
    nr = rays.shape[0] * rays.shape[1]
    S, start, g = _setup(s, rays, half)
    dq = _quantiles(nr, np.random.default_rng(1))
    ref = oracle.trace_fwd(S, rays, start, depth_quantiles=dq, wt=0.01, return_contribution=True,
                           seq_cap=SEQ)
    dbg = {"seq_cap": SEQ}
    out = _ops.trace_vorotracing_fwd(g["points"], g["diffuse"], g["specular"], g["density"],
                                     g["adj"], g["offs"], _dev(rays), _dev(start).view(rays.shape[:2]),
                                     _dev(dq).view(*rays.shape[:2], 3), 0.01, 1024, True,
                                     debug=dbg)
    torch.cuda.synchronize()
    rgba, depth, didx, contrib, n_int, dist, W, S_, tfar = out
    np.testing.assert_array_equal(dbg["seq"].cpu().numpy(), ref["seq"].astype(np.int32))
    np.testing.assert_array_equal(n_int.cpu().numpy().reshape(-1).astype(np.int64),
                                  ref["n"].astype(np.int64))
    if half:
        np.testing.assert_array_equal(rgba.cpu().numpy().reshape(-1, 4).view(np.uint16),
                                      ref["rgba"].view(np.uint16))
    else:
        np.testing.assert_array_equal(rgba.cpu().numpy().reshape(-1, 4), ref["rgba"])
    np.testing.assert_array_equal(depth.cpu().numpy().reshape(-1, 3), ref["depth"])
    np.testing.assert_array_equal(didx.cpu().numpy().reshape(-1, 3).astype(np.int64),
                                  ref["depth_idx"].astype(np.int64))
    for a, b in ((dist, "distortion"), (W, "W"), (S_, "S"), (tfar, "t_far")):
        np.testing.assert_array_equal(a.cpu().numpy().reshape(-1), ref[b])
    c = contrib.float().cpu().numpy().reshape(-1)
    if half:
        # binary16 atomics (as in the reference) stagnate once a running sum's
        # ulp exceeds the added weights; the oracle sums in binary32
        np.testing.assert_allclose(c, ref["contribution"], rtol=1e-1, atol=5e-3)
    else:
        np.testing.assert_allclose(c, ref["contribution"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("with_extras", [False, True])
@pytest.mark.parametrize("path_cap", [None, 1, 7, 1024])
def test_bwd_matches_oracle(c1_scene, c1_rays, half, with_extras, path_cap):
    """path_cap: the backward replays the forward's path record (cap steps
    per ray, the face scan resuming after them) instead of walking."""
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    rays = c1_rays[::2, ::2].reshape(-1, 6)
    nr = rays.shape[0]
    rng = np.random.default_rng(2)
    S, start, g = _setup(s, rays, half)
    dq = _quantiles(nr, rng) if with_extras else None
    f = oracle.trace_fwd(S, rays, start, depth_quantiles=dq, wt=0.01)
    adt = np.float16 if half else np.float32
    rgba = np.asarray(f["rgba"]).astype(adt)
    grgba = rng.normal(0, 1, (nr, 4)).astype(adt)
    kw = {}
    if with_extras:
        kw = dict(depth_quantiles=dq, depth_idx=f["depth_idx"],
                  depth_grad=rng.normal(0, 1, (nr, 3)).astype(np.float32),
                  ray_error=rng.uniform(0, 1, nr).astype(adt), contribution_alpha_grad=0.25,
                  distortion=f["distortion"], distortion_grad=rng.normal(0, 1, nr).astype(np.float32))
    ref = oracle.trace_bwd(S, rays, start, rgba, grgba, W=f["W"], S=f["S"], t_far=f["t_far"],
                           wt=0.01, **{k: v for k, v in kw.items() if k != "distortion"},
                           distortion=f["distortion"])
    t = lambda a: None if a is None else _dev(a)
    path = None
    if path_cap is not None:
        path = _ops.PathRecord(nr, path_cap, "cuda")
        _ops.trace_vorotracing_fwd(g["points"], g["diffuse"], g["specular"], g["density"],
                                   g["adj"], g["offs"], _dev(rays), _dev(start), t(dq), 0.01, 1024,
                                   False, path=path)
    res = _ops.trace_vorotracing_bwd(
        g["points"], g["diffuse"], g["specular"], g["density"], g["adj"], g["offs"], _dev(rays),
        _dev(start), _dev(rgba), _dev(grgba), t(dq), t(kw.get("depth_idx")),
        t(kw.get("depth_grad")), t(kw.get("ray_error")), kw.get("contribution_alpha_grad", 0.0),
        _dev(f["distortion"]), t(kw.get("distortion_grad")), _dev(f["W"]), _dev(f["S"]),
        _dev(f["t_far"]), 0.01, 1024, path=path)
    torch.cuda.synchronize()
    pg, dg, sg, deng, _, perr = res
    # fp16 attributes: the texel / point-error gradients are summed in fp32
    # workspace and rounded to binary16 once, like the oracle's fp32 sums
    # rounded here: one binary16 ulp apart at most
    _close(pg.cpu().numpy(), ref["points"], 1e-3, 1e-4, "points")
    _close(deng.cpu().numpy().reshape(-1), ref["density"], 1e-3, 1e-4, "density")
    near = close_f16 if half else (lambda a, b, name: _close(a, b, 1e-3, 1e-4, name))
    near(dg.float().cpu().numpy(), ref["diffuse"], "diffuse")
    near(sg.float().cpu().numpy(), ref["specular"], "specular")
    if with_extras:
        near(perr.float().cpu().numpy().reshape(-1), ref["point_error"], "point_error")
    else:
        assert perr is None


def test_autograd_function(c1_scene, c1_rays):
    from vorotracing_b200.cuda import TraceVoroTracing, _ops

    s = c1_scene
    rays = _dev(c1_rays[::4, ::4])
    S, start, g = _setup(s, c1_rays[::4, ::4], False)
    params = [g["points"].clone().requires_grad_(), g["diffuse"].clone().requires_grad_(),
              g["specular"].clone().requires_grad_(), g["density"].clone().requires_grad_()]
    st = _dev(start).view(rays.shape[:2])
    rgba, depth, contrib, n_int, errbox, dist = TraceVoroTracing.apply(
        *params, g["adj"], g["offs"], rays, st, None, 0.01, 1024, False)
    target = torch.rand_like(rgba)
    loss = ((rgba - target) ** 2).mean() + 0.01 * dist.mean()
    loss.backward()
    f = _ops.trace_vorotracing_fwd(*[p.detach() for p in params], g["adj"], g["offs"], rays, st,
                                   None, 0.01, 1024, False)
    grad_rgba = 2.0 * (f[0] - target) / rgba.numel()
    grad_dist = torch.full_like(f[5], 0.01 / dist.numel())
    ref = _ops.trace_vorotracing_bwd(*[p.detach() for p in params], g["adj"], g["offs"], rays, st,
                                     f[0], grad_rgba, None, None, None, None, 0.0, f[5], grad_dist,
                                     f[6], f[7], f[8], 0.01, 1024)
    for p, r in zip(params, ref[:4]):
        torch.testing.assert_close(p.grad, torch.nan_to_num(r), rtol=1e-4, atol=1e-7)
    assert depth is None and contrib is None and isinstance(errbox.ray_error, type(None))


def test_fwd_validation_messages(c1_scene, c1_rays):
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    S, start, g = _setup(s, c1_rays[:2, :2], False)
    rays = _dev(c1_rays[:2, :2])
    with pytest.raises(RuntimeError, match="start_point must have uint32 dtype"):
        _ops.trace_vorotracing_fwd(g["points"], g["diffuse"], g["specular"], g["density"],
                                   g["adj"], g["offs"], rays, _dev(start.astype(np.int32)), None,
                                   0.01, 1024, False)
    with pytest.raises(RuntimeError, match="same dtype"):
        _ops.trace_vorotracing_fwd(g["points"], g["diffuse"], g["specular"].half(), g["density"],
                                   g["adj"], g["offs"], rays, _dev(start), None, 0.01, 1024, False)


def test_bwd_into_flat_bucket(c1_scene, c1_rays):
    """The backward writes into caller-provided views of one flat all-reduce
    bucket with the same result as into its own tensors."""
    from vorotracing_b200.cuda import _ops
    from vorotracing_b200.shard import GradBucket

    s = c1_scene
    rays = c1_rays[::4, ::4].reshape(-1, 6)
    S, start, g = _setup(s, rays, False)
    args = (g["points"], g["diffuse"], g["specular"], g["density"], g["adj"], g["offs"],
            _dev(rays), _dev(start))
    f = _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False)
    gr = torch.randn_like(f[0])
    common = (f[0], gr, None, None, None, None, 0.0, f[5], None, f[6], f[7], f[8], 0.01, 1024)
    ref = _ops.trace_vorotracing_bwd(*args, *common)
    b = GradBucket(g["points"].size(0), g["diffuse"].size(1), "cuda")
    _ops.trace_vorotracing_bwd(*args, *common, grads=b.views())
    # same kernels, different destination: equal up to the order of the fp32
    # atomic additions (sums of many terms with cancellation)
    for got, want in zip(b.views(), (ref[0], ref[1], ref[2], ref[3])):
        scale = float(want.abs().max()) if want.numel() else 1.0
        torch.testing.assert_close(got.reshape(want.shape), want, rtol=1e-4, atol=1e-5 * scale)
    # overwrite mode: the bucket's previous contents do not matter
    b.flat.fill_(123.0)
    _ops.trace_vorotracing_bwd(*args, *common, grads=b.views(), accumulate=False)
    for got, want in zip(b.views(), (ref[0], ref[1], ref[2], ref[3])):
        scale = float(want.abs().max()) if want.numel() else 1.0
        torch.testing.assert_close(got.reshape(want.shape), want, rtol=1e-4, atol=1e-5 * scale)
    # no rays: overwriting leaves zero gradients
    b.flat.fill_(123.0)
    empty = lambda t: t[:0]
    _ops.trace_vorotracing_bwd(*args[:6], empty(args[6]), empty(args[7]), empty(f[0]),
                               empty(gr), None, None, None, None, 0.0, empty(f[5]), None,
                               empty(f[6]), empty(f[7]), empty(f[8]), 0.01, 1024,
                               grads=b.views(), accumulate=False)
    assert not b.flat.any()


@pytest.mark.parametrize("half", [False, True])
def test_bwd_vector_atomics_match_scalar(c1_scene, c1_rays, half):
    """Padded-scratch vector atomics and scalar atomics into the outputs give
    the same gradients (up to summation order; fp16 is summed in fp32 first)."""
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    rays = c1_rays[::2, ::2].reshape(-1, 6)
    S, start, g = _setup(s, rays, half)
    args = (g["points"], g["diffuse"], g["specular"], g["density"], g["adj"], g["offs"],
            _dev(rays), _dev(start))
    f = _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False)
    gr = torch.randn_like(f[0].float()).to(f[0].dtype)
    common = (f[0], gr, None, None, None, None, 0.0, f[5], None, f[6], f[7], f[8], 0.01, 1024)
    a = _ops.trace_vorotracing_bwd(*args, *common, vector_atomics=True)
    b = _ops.trace_vorotracing_bwd(*args, *common, vector_atomics=False)
    for x, y, name in zip(a[:4], b[:4], ("points", "diffuse", "specular", "density")):
        tol, frac = (1e-1, 2e-2) if half and name in ("diffuse", "specular") else (1e-3, 1e-4)
        _close(x.float().cpu().numpy(), y.float().cpu().numpy(), tol, frac, name)


@pytest.mark.parametrize("cap", [1, 5, 1024])
def test_path_record_is_the_cell_sequence(c1_scene, c1_rays, cap):
    """The forward's path record holds the cells entered at each step (the
    visited-cell sequence shifted by one) and the number of exit faces found."""
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    rays = c1_rays[::2, ::2].reshape(-1, 6)
    nr = rays.shape[0]
    S, start, g = _setup(s, rays, False)
    args = (g["points"], g["diffuse"], g["specular"], g["density"], g["adj"], g["offs"],
            _dev(rays), _dev(start))
    path = _ops.PathRecord(nr, cap, "cuda")
    dbg = {"seq_cap": SEQ}
    _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False, path=path, debug=dbg)
    seq = dbg["seq"].cpu().numpy().reshape(nr, SEQ)
    seq_len = dbg["seq_len"].cpu().numpy().reshape(-1)
    cells = path.cells.cpu().numpy()
    plen_raw = path.len.cpu().numpy()
    plen = plen_raw & 0x7FFFFFFF
    # the high bit asks the backward to walk the ray itself (record overflow)
    assert np.all(((plen_raw >> 31) == 1) >= (plen > cap))
    ref = oracle.trace_fwd(S, rays, start, wt=0.01, seq_cap=SEQ)
    # the walk ends on a cell with no exit face, or stops integrating inside one
    assert np.all((plen == seq_len) | (plen == seq_len - 1))
    for r in range(nr):
        # the exit neighbour of the last step is recorded but never entered
        m = min(int(plen[r]), cap, int(seq_len[r]) - 1, SEQ - 1)
        np.testing.assert_array_equal(cells[:m, r], seq[r, 1:m + 1])
    assert np.array_equal(seq_len, np.asarray(ref["seq_len"]).reshape(-1))
