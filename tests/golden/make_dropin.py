"""Record the operator calls the reference's own model code makes.

    python tests/golden/make_dropin.py /path/to/VoroTracing

Imports the reference's ``vorotracing.vorotracing`` (VoroTracing,
VoroTracingInfer; vorotracing/vorotracing.py) with ``vorotracing.cuda``
replaced by a recording module whose operators are computed by this
repository's CPU oracle (oracle/, the tests' checker), then drives the model
code as the trainer and the viewer do:

  VoroTracing.forward + loss.backward     vorotracing.py:365-419 (start cell :323-344,
                                          activation :346-347), with depth quantiles,
                                          contribution, ray error and, in a second
                                          step, cell_distortion_gate (_wrapper.py:145-171)
  VoroTracingInfer(..., "fp16").render    vorotracing.py:439-493, 627-683 (Morton reorder,
                                          _pad_3to4, prefetch_octmap_adj, 4x8 tile perm)
  VoroTracingInfer(..., "q8").render      the same with _quantize_to_uint8

Every argument the model code passes to an operator, the upstream gradients
autograd hands to the backward, and the operators' (oracle) results are
written to tests/golden/dropin_calls.npz.  tests/test_gpu_dropin.py replays
those exact calls through ``vorotracing_b200.cuda`` on the GPU.  The large
texture arrays are not stored: they are regenerated from the seed below
(``scene_inputs``) and checked against recorded SHA-256 digests.
"""
from __future__ import annotations

import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "dropin_calls.npz")

N_SITES, RES, W, H, SEED = 1024, 8, 32, 24, 2024


def sha(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


def scene_inputs():
    """Seeded model inputs (numpy only, so the GPU test regenerates them):
    sites on a noisy sphere plus uniform ones, texture logits, density logits."""
    rng = np.random.default_rng(SEED)
    m = int(N_SITES * 0.7)
    d = rng.standard_normal((m, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    surf = d * (1.0 + 0.01 * rng.standard_normal((m, 1)))
    uni = rng.uniform(-2, 2, (N_SITES - m, 3))
    pts = np.concatenate([surf, uni]).astype(np.float32)
    diffuse = rng.normal(0.0, 1.0, (N_SITES, 3 * RES * RES)).astype(np.float32)
    specular = rng.normal(0.0, 0.3, (N_SITES, 3 * RES * RES)).astype(np.float32)
    density = rng.normal(0.5, 1.0, (N_SITES, 1)).astype(np.float32)
    return pts, diffuse, specular, density


def _rays():
    sys.path.insert(0, ROOT)
    from vorotracing_b200.scene import intrinsics, look_at, pinhole_rays

    return pinhole_rays(intrinsics(W, H), look_at((0.3, -2.8, 0.9)), W, H)


def _recording_ops(rec: dict):
    import oracle

    ops = types.ModuleType("vorotracing.cuda")
    n_calls = {}

    def key(name):
        i = n_calls.get(name, 0)
        n_calls[name] = i + 1
        return f"{name}{i}"

    def put(k, name, v):
        if isinstance(v, torch.Tensor):
            v = v.detach().numpy()
        rec[f"{k}.{name}"] = np.asarray(v)

    def np_(t):
        return t.detach().contiguous().numpy()

    def attr_kind(t):
        return {torch.float32: oracle.ATTR_F32, torch.float16: oracle.ATTR_F16}[t.dtype]

    class NNBVH:
        def build(self, points):
            self.n = points.shape[0]

        def query(self, points, queries):
            k = key("bvh_query")
            put(k, "points_sha", sha(np_(points)))
            put(k, "queries", queries)
            out = torch.from_numpy(oracle.nn_query(np_(points), np_(queries)))
            put(k, "out", out)
            return out

    class ErrorBox:
        def __init__(self):
            self.ray_error = None
            self.point_error = None
            self.cell_distortion_gate = None

    class TraceVoroTracing(torch.autograd.Function):
        @staticmethod
        def forward(ctx, points, diffuse, specular, density, adj, offs, rays, start_point,
                    depth_quantiles, weight_threshold, max_intersections, return_contribution):
            k = key("train")
            ctx.k = k
            for name, t in (("points", points), ("density", density), ("adjacency", adj),
                            ("offsets", offs), ("rays", rays), ("start_point", start_point)):
                put(k, name, t)
            put(k, "diffuse_sha", sha(np_(diffuse)))
            put(k, "specular_sha", sha(np_(specular)))
            put(k, "diffuse_dtype", str(diffuse.dtype))
            if depth_quantiles is not None:
                put(k, "depth_quantiles", depth_quantiles)
            put(k, "scalars", np.array([weight_threshold, max_intersections,
                                        float(return_contribution)], np.float64))
            S = oracle.Scene(np_(points), np_(adj), np_(offs), np_(density), np_(diffuse),
                             np_(specular), attr_kind(diffuse))
            nr = rays.numel() // 6
            dq = None if depth_quantiles is None else np_(depth_quantiles).reshape(nr, -1)
            f = oracle.trace_fwd(S, np_(rays), np_(start_point).reshape(-1), depth_quantiles=dq,
                                 wt=weight_threshold, max_int=max_intersections,
                                 return_contribution=bool(return_contribution))
            lead = tuple(rays.shape[:-1])
            rgba = torch.from_numpy(np.ascontiguousarray(f["rgba"])).reshape(lead + (4,))
            depth = None if dq is None else torch.from_numpy(f["depth"].copy()).reshape(lead + (-1,))
            contrib = (torch.from_numpy(f["contribution"]).reshape(-1, 1)
                       if return_contribution else None)
            n_int = torch.from_numpy(f["n"].astype(np.int64)).reshape(lead + (1,))
            dist = torch.from_numpy(f["distortion"]).reshape(lead + (1,))
            for name in ("rgba", "depth", "contribution", "distortion", "n"):
                if f.get(name) is not None:
                    put(k, "out_" + name, f[name])
            ctx.S, ctx.f, ctx.dq = S, f, dq
            ctx.args = (np_(rays).reshape(-1, 6), np_(start_point).reshape(-1), weight_threshold,
                        max_intersections)
            errbox = ErrorBox()
            ctx.errbox = errbox
            ctx.mark_non_differentiable(n_int)
            return rgba, depth, contrib, n_int, errbox, dist

        @staticmethod
        def backward(ctx, grad_rgba, grad_depth, grad_contribution, grad_n, errbox_grad,
                     grad_distortion):
            k = ctx.k
            S, f, dq = ctx.S, ctx.f, ctx.dq
            rays, start, wt, mi = ctx.args
            cag = 0.0 if grad_contribution is None else float(grad_contribution.abs().max())
            put(k, "grad_rgba", grad_rgba)
            if grad_depth is not None:
                put(k, "grad_depth", grad_depth)
            if grad_contribution is not None:
                put(k, "grad_contribution", grad_contribution)
            if grad_distortion is not None:
                put(k, "grad_distortion", grad_distortion)
            re = ctx.errbox.ray_error
            gate = ctx.errbox.cell_distortion_gate
            if re is not None:
                put(k, "ray_error", re)
            if gate is not None:
                put(k, "cell_distortion_gate", gate)
            nr = rays.shape[0]

            def bwd(g_rgba, g_depth, ray_error, contrib, g_dist):
                return oracle.trace_bwd(
                    S, rays, start, f["rgba"], g_rgba.reshape(nr, 4), depth_quantiles=dq,
                    depth_idx=None if dq is None else f["depth_idx"],
                    depth_grad=None if dq is None else g_depth.reshape(nr, -1),
                    ray_error=None if ray_error is None else ray_error.reshape(-1),
                    contribution_alpha_grad=contrib, distortion=f["distortion"],
                    distortion_grad=None if g_dist is None else g_dist.reshape(-1),
                    W=f["W"], S=f["S"], t_far=f["t_far"], wt=wt, max_int=mi)

            g_rgba = np_(grad_rgba)
            g_depth = None if grad_depth is None else np_(grad_depth)
            g_dist = None if grad_distortion is None else np_(grad_distortion)
            rerr = None if re is None else np_(re)
            if gate is not None and g_dist is not None:
                rd = bwd(np.zeros_like(g_rgba), None if g_depth is None else np.zeros_like(g_depth),
                         None, 0.0, g_dist)
                r = bwd(g_rgba, g_depth, rerr, cag, np.zeros_like(g_dist))
                r["density"] = r["density"] + np_(gate).reshape(-1) * np.nan_to_num(rd["density"])
            else:
                r = bwd(g_rgba, g_depth, rerr, cag, g_dist)
            out = [np.nan_to_num(r[n]) for n in ("points", "diffuse", "specular", "density")]
            for n, a in zip(("points", "diffuse", "specular", "density"), out):
                put(k, "grad_out_" + n, a)
            if r.get("point_error") is not None:
                put(k, "point_error", r["point_error"])
            ctx.errbox.point_error = (None if r.get("point_error") is None
                                      else torch.from_numpy(r["point_error"]).reshape(-1, 1))
            shapes = (S.points.shape, S.diffuse.shape, S.specular.shape, (S.points.shape[0], 1))
            grads = [torch.from_numpy(a.reshape(s).astype(np.float32)) for a, s in zip(out, shapes)]
            return (*grads, None, None, None, None, None, None, None, None)

    def prefetch_octmap_adj(points, adjacency, offsets):
        k = key("prefetch")
        for name, t in (("points", points), ("adjacency", adjacency), ("offsets", offsets)):
            put(k, name, t)
        out = oracle.prefetch_adj(np_(points), np_(adjacency), np_(offsets))
        put(k, "out", out)
        return torch.from_numpy(out).view(torch.float16)

    def _infer(kind, points, diffuse, specular, density, adjacency, offsets, rays, start_point,
               adjacent_diff, ray_perm, q8, weight_threshold, max_intersections,
               cell_skip_threshold):
        k = key(kind)
        for name, t in (("points", points), ("density", density), ("adjacency", adjacency),
                        ("offsets", offsets), ("rays", rays), ("start_point", start_point),
                        ("adjacent_diff", adjacent_diff.view(torch.int16))):
            put(k, name, t)
        put(k, "diffuse_sha", sha(np_(diffuse)))
        put(k, "specular_sha", sha(np_(specular)))
        if ray_perm is not None:
            put(k, "ray_perm", ray_perm)
        if q8 is not None:
            put(k, "q8", np.array(q8, np.float64))
        put(k, "scalars", np.array([weight_threshold, max_intersections, cell_skip_threshold],
                                   np.float64))
        attr = oracle.ATTR_U8 if q8 is not None else oracle.ATTR_F16X4
        dfn = np_(diffuse) if q8 is not None else np_(diffuse.view(torch.int16)).view(np.uint16)
        sfn = np_(specular) if q8 is not None else np_(specular.view(torch.int16)).view(np.uint16)
        S = oracle.Scene(np_(points), np_(adjacency), np_(offsets), np_(density), dfn, sfn, attr,
                         q8=tuple(np.float32(v) for v in q8) if q8 is not None else
                         (1.0, 0.0, 1.0, 0.0))
        r = oracle.trace_infer(S, np_(rays), np_(start_point).reshape(-1), wt=weight_threshold,
                               max_int=max_intersections, skip=cell_skip_threshold)
        put(k, "out_rgba", r["rgba"].view(np.uint16))
        return torch.from_numpy(r["rgba"].copy()).reshape(tuple(rays.shape[:-1]) + (4,))

    def trace_octmap_infer(points, diffuse_fp16, specular_fp16, density, adjacency, offsets, rays,
                           start_point, adjacent_diff, ray_perm, weight_threshold=0.001,
                           max_intersections=1024, cell_skip_threshold=0.0):
        return _infer("infer_f16_", points, diffuse_fp16, specular_fp16, density, adjacency,
                      offsets, rays, start_point, adjacent_diff, ray_perm, None,
                      weight_threshold, max_intersections, cell_skip_threshold)

    def trace_octmap_infer_q8(points, diffuse_q8, specular_q8, density, adjacency, offsets, rays,
                              start_point, adjacent_diff, diff_scale, diff_offset, spec_scale,
                              spec_offset, weight_threshold=0.001, max_intersections=1024,
                              cell_skip_threshold=0.0):
        return _infer("infer_q8_", points, diffuse_q8, specular_q8, density, adjacency, offsets,
                      rays, start_point, adjacent_diff, None,
                      (diff_scale, diff_offset, spec_scale, spec_offset), weight_threshold,
                      max_intersections, cell_skip_threshold)

    ops.NNBVH = NNBVH
    ops.ErrorBox = ErrorBox
    ops.TraceVoroTracing = TraceVoroTracing
    ops.prefetch_octmap_adj = prefetch_octmap_adj
    ops.trace_octmap_infer = trace_octmap_infer
    ops.trace_octmap_infer_q8 = trace_octmap_infer_q8
    return ops


def main(ref_root: str):
    sys.path.insert(0, ROOT)
    rec = {}
    sys.modules["vorotracing.cuda"] = _recording_ops(rec)
    sys.path.insert(0, ref_root)
    import vorotracing.vorotracing as vv
    from scipy.spatial import Delaunay

    pts, dif, spe, den = scene_inputs()
    ip, ind = Delaunay(pts.astype(np.float64)).vertex_neighbor_vertices
    adj = np.zeros(len(ind) + 32, np.uint32)
    adj[: len(ind)] = ind
    offs = ip.astype(np.uint32)
    rec["scene.adjacency"] = adj
    rec["scene.offsets"] = offs
    rec["scene.sha"] = np.array([sha(pts), sha(dif), sha(spe), sha(den)])

    cfg = vv.VoroTracingConfig()
    assert cfg.oct_map_res == RES and cfg.spec_oct_map_res == RES
    cpu = torch.device("cpu")
    model = vv.VoroTracing(cfg, torch.from_numpy(pts), torch.from_numpy(dif),
                           torch.from_numpy(spe), torch.from_numpy(den),
                           torch.from_numpy(adj.astype(np.int64)),
                           torch.from_numpy(offs.astype(np.int64)), device=cpu)
    rays = torch.from_numpy(_rays())
    rng = np.random.default_rng(SEED + 1)
    target = torch.from_numpy(rng.uniform(0, 1, (H, W, 3)).astype(np.float32))
    dq = torch.from_numpy(np.sort(rng.uniform(0.1, 0.9, (H, W, 2)).astype(np.float32),
                                  axis=-1)[..., ::-1].copy())
    ray_err = torch.from_numpy(rng.uniform(0, 1, (H, W)).astype(np.float32))
    gate = torch.from_numpy(rng.uniform(0, 2, (N_SITES, 1)).astype(np.float32))
    for step in range(2):
        model.zero_grad()
        rgba, depth, contrib, n_int, errbox, dist = model(rays, depth_quantiles=dq,
                                                          weight_threshold=0.01,
                                                          return_contribution=True)
        errbox.ray_error = ray_err
        if step == 1:
            errbox.cell_distortion_gate = gate
        loss = (((rgba[..., :3] - target) ** 2).mean() + 0.01 * dist.mean()
                + 1e-3 * depth.mean() + 0.1 * contrib.sum())
        loss.backward()
        rec[f"train{step}.param_grad_density"] = model.density.grad.numpy().copy()

    for q in ("fp16", "q8"):
        inf = vv.VoroTracingInfer(model, sort_morton=True, quantize=q)
        inf.render(rays, weight_threshold=0.01, cell_skip_threshold=1e-3)
        # the Morton permutation, so the test can rebuild the sorted textures
        order = {tuple(p): i for i, p in enumerate(pts.tolist())}
        perm = np.array([order[tuple(p)] for p in inf.primal_points.numpy().tolist()], np.int64)
        rec[f"morton_perm_{q}"] = perm
    np.savez_compressed(OUT, **rec)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len(rec), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
