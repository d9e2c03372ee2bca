"""How far the reference's fast-math arithmetic moves traversals and pixels.

The reference extension is compiled with -use_fast_math and contraction on
(vorotracing/cuda/_backend.py:188-204): approximate division, CUDA's fast
expf / logf, fused multiply-adds where the compiler chooses.  This package's
kernels (and the oracle) use exact IEEE operations, so bit-exact parity with
the oracle does not by itself say how close they are to the reference binary,
which cannot be built here.  ``libvorotracing_b200_refmath.so`` is the same
source compiled with the reference's flags and the reference's expression
shapes (``d /= len`` in the probe direction, ray_integrator_octmap.cuh:
703-704; ``expf`` / ``logf`` for the exponentials).  These tests render the
same inputs with both builds and bound the differences:

* the fraction of rays whose visited-cell sequence differs, and of rays whose
  first exit face (the first cell entered) differs;
* the largest and the 99.9th-percentile |delta rgb| of the fp16 inference
  pixels and of the fp32 training forward.

Set VT_REFMATH_REPORT=<file> to have the measured rates written as JSON.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

SEQ = 256
REPORT = {}


@pytest.fixture(scope="module")
def refmath_lib():
    from vorotracing_b200 import _lib
    from vorotracing_b200 import build as b

    if not os.path.exists(b.LIB_REFMATH):
        b.build(refmath=True)
    yield _lib.load(b.LIB_REFMATH, require_all=False)
    path = os.environ.get("VT_REFMATH_REPORT")
    if path:
        with open(path, "w") as f:
            json.dump(REPORT, f, indent=1)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _seq_stats(sa, la, sb, lb):
    n = sa.shape[0]
    cap = sa.shape[1]
    la = np.minimum(la, cap)
    lb = np.minimum(lb, cap)
    idx = np.arange(cap)[None, :]
    ma = np.where(idx < la[:, None], sa, -1)
    mb = np.where(idx < lb[:, None], sb, -1)
    differ = (ma != mb).any(1) | (la != lb)
    first = (ma[:, 1] != mb[:, 1]) if cap > 1 else np.zeros(n, bool)
    return float(differ.mean()), float(first.mean())


def _pix_stats(a, b):
    d = np.abs(np.asarray(a, np.float64)[..., :3] - np.asarray(b, np.float64)[..., :3]).reshape(-1)
    return float(d.max()), float(np.quantile(d, 0.999)), float(d.mean())


def _infer_both(L, scene_t, rays, start, res):
    from vorotracing_b200 import _lib
    from vorotracing_b200.cuda import _ops

    pts, dif, spe, den, adj, offs = scene_t
    out = []
    for lib in (None, L):
        dbg = {"seq_cap": SEQ}
        if lib is None:
            faces = _ops.prefetch_faces(pts, adj, offs)
            rgba = _ops.trace_vorotracing_infer(pts, dif, spe, den, adj, offs, rays, start, faces,
                                                None, 0.01, 1024, 1e-3, debug=dbg)
        else:
            with _lib.using(lib):
                faces = _ops.prefetch_faces(pts, adj, offs)
                rgba = _ops.trace_vorotracing_infer(pts, dif, spe, den, adj, offs, rays, start,
                                                    faces, None, 0.01, 1024, 1e-3, debug=dbg)
        torch.cuda.synchronize()
        out.append((rgba.float().cpu().numpy(), dbg["seq"].cpu().numpy(),
                    dbg["seq_len"].cpu().numpy()))
    return out


def test_refmath_c1_infer(refmath_lib, c1_scene, c1_rays):
    s = c1_scene
    res = s["res"]
    t = (_dev(s["points"]), _dev(oracle.pad_f16x4(s["diffuse"], res)),
         _dev(oracle.pad_f16x4(s["specular"], res)), _dev(s["density"]), _dev(s["adj"]),
         _dev(s["offs"]))
    st = oracle.nn_query(s["points"], c1_rays.reshape(-1, 6)[:1, :3])[0]
    start = _dev(np.full(c1_rays.shape[0] * c1_rays.shape[1], st, np.uint32))
    (ra, sa, la), (rb, sb, lb) = _infer_both(refmath_lib, t, _dev(c1_rays), start, res)
    seq_frac, first_frac = _seq_stats(sa, la, sb, lb)
    mx, p999, mean = _pix_stats(ra, rb)
    REPORT["c1_infer_f16"] = dict(rays=int(len(la)), seq_differ=seq_frac,
                                  first_exit_differ=first_frac, max_drgb=mx, p999_drgb=p999,
                                  mean_drgb=mean)
    # the exact build is the oracle's (checked elsewhere); the fast-math build
    # must stay close to it
    assert first_frac <= 0.01
    assert seq_frac <= 0.05
    assert p999 <= 2e-2 and mx <= 0.5


def test_refmath_c2_infer(refmath_lib):
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.render import InferScene

    s = sc.config_scene("C2", adjacency="gpu", cache=False)
    scene = InferScene(_dev(s["points"]), _dev(s["density"]), _dev(s["adj"]), _dev(s["offs"]),
                       _dev(s["diffuse"]), _dev(s["specular"]), quantize="fp16")
    rays_np = sc.config_rays("C2")
    rays = _dev(rays_np)
    start = scene.get_starting_point(rays).reshape(-1).contiguous()
    t = (scene.primal_points, scene.diffuse_fp16, scene.specular_fp16, scene.density,
         scene.point_adjacency, scene.point_adjacency_offsets)
    (ra, sa, la), (rb, sb, lb) = _infer_both(refmath_lib, t, rays, start, 8)
    seq_frac, first_frac = _seq_stats(sa, la, sb, lb)
    mx, p999, mean = _pix_stats(ra, rb)
    REPORT["c2_infer_f16"] = dict(rays=int(len(la)), seq_differ=seq_frac,
                                  first_exit_differ=first_frac, max_drgb=mx, p999_drgb=p999,
                                  mean_drgb=mean, seq_cap=SEQ)
    assert first_frac <= 0.01
    assert seq_frac <= 0.1
    assert p999 <= 5e-2


def test_refmath_c1_train_fwd(refmath_lib, c1_scene, c1_rays):
    from vorotracing_b200 import _lib
    from vorotracing_b200.cuda import _ops

    s = c1_scene
    rays = _dev(c1_rays.reshape(-1, 6))
    st = oracle.nn_query(s["points"], c1_rays.reshape(-1, 6)[:1, :3])[0]
    start = _dev(np.full(rays.size(0), st, np.uint32))
    args = (_dev(s["points"]), _dev(s["diffuse"]), _dev(s["specular"]), _dev(s["density"]),
            _dev(s["adj"]), _dev(s["offs"]), rays, start, None, 0.01, 1024, False)
    a = _ops.trace_vorotracing_fwd(*args)
    with _lib.using(refmath_lib):
        b = _ops.trace_vorotracing_fwd(*args)
    torch.cuda.synchronize()
    mx, p999, mean = _pix_stats(a[0].cpu().numpy(), b[0].cpu().numpy())
    nd = float((a[4] != b[4]).float().mean())
    REPORT["c1_train_fwd_f32"] = dict(rays=int(rays.size(0)), steps_differ=nd, max_drgb=mx,
                                      p999_drgb=p999, mean_drgb=mean)
    assert nd <= 0.05
    assert p999 <= 2e-2
