"""Generate golden vectors from the reference's own Python code.

    python tests/golden/make_golden.py /path/to/VoroTracing

Runs, on CPU torch and on small seeded inputs, the reference functions that
define the layout transforms and the camera convention of the hot path:

  VoroTracingInfer._tile_perm          vorotracing/vorotracing.py:606-625
  VoroTracingInfer._quantize_to_uint8  vorotracing/vorotracing.py:495-503
  VoroTracingInfer._pad_3to4           vorotracing/vorotracing.py:505-512
  VoroTracingInfer._reorder_by_morton  vorotracing/vorotracing.py:514-571
  generate_camera_rays                 vorotracing/utils/__init__.py:85-130
  write_foam (.foam V4 and V3)         scripts/export_for_viewer.py:146-216
  VoroTracing.save_checkpoint          vorotracing/vorotracing.py:421-436

The reference's compiled extension is replaced by a stub module (its import
would JIT-compile CUDA code that cannot be built here); none of the functions
above call into it except NNBVH.build, which the stub makes a no-op.
Outputs (committed): tests/golden/layout_golden.npz, and scene_v4.foam /
scene_v3.foam with their inputs in foam_inputs.npz.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    stub = types.ModuleType("vorotracing.cuda")

    class _NoBVH:
        def build(self, points):
            pass

    stub.NNBVH = _NoBVH
    sys.modules["vorotracing.cuda"] = stub
    sys.path.insert(0, root)
    import vorotracing.vorotracing as vv
    import vorotracing.utils as vu

    return vv, vu


def main(root: str):
    vv, vu = _import_reference(root)
    Infer = vv.VoroTracingInfer
    out = {}
    rng = np.random.default_rng(123)

    # tile permutation, including ragged edge tiles
    for H, W in [(8, 16), (13, 21), (37, 45), (5, 3)]:
        obj = object.__new__(Infer)
        obj.primal_points = torch.zeros(1, 3)
        out[f"tile_{H}x{W}"] = Infer._tile_perm(obj, H, W).numpy()

    # quantisation and fp16 padding
    tex = torch.from_numpy(rng.normal(0.0, 1.5, (257, 3 * 64)).astype(np.float32))
    q, scale, offset = Infer._quantize_to_uint8(tex)
    out["quant_src"] = tex.numpy()
    out["quant_q"] = q.numpy()
    out["quant_scale_offset"] = np.array([scale, offset], np.float64)
    out["pad_src"] = tex.numpy()
    out["pad_out"] = Infer._pad_3to4(tex.half(), 8).view(torch.int16).numpy()

    # Morton reorder of sites and CSR (the codes have no ties in this sample,
    # so the reference's unstable argsort is deterministic here)
    n = 3000
    pts = rng.uniform(-2, 2, (n, 3)).astype(np.float32)
    from scipy.spatial import Delaunay

    ip, ind = Delaunay(pts.astype(np.float64)).vertex_neighbor_vertices
    adj = np.zeros(len(ind) + 32, np.int64)
    adj[: len(ind)] = ind
    obj = object.__new__(Infer)
    obj.primal_points = torch.from_numpy(pts)
    obj.density = torch.from_numpy(rng.uniform(0, 1, (n, 1)).astype(np.float32))
    obj.quantize = "fp16"
    obj.diffuse_fp16 = torch.from_numpy(rng.normal(size=(n, 8)).astype(np.float16))
    obj.specular_fp16 = obj.diffuse_fp16.clone()
    obj.point_adjacency = torch.from_numpy(adj)
    obj.point_adjacency_offsets = torch.from_numpy(ip.astype(np.int64))
    obj.bvh = sys.modules["vorotracing.cuda"].NNBVH()
    # codes as the reference computes them (vorotracing.py:519-530)
    bmin = obj.primal_points.min(dim=0).values
    bmax = obj.primal_points.max(dim=0).values
    size = (bmax - bmin).clamp(min=1e-6)
    norm = ((obj.primal_points - bmin) / size * 1023.0).clamp(0, 1023).long()
    code = torch.zeros(n, dtype=torch.long)
    for i in range(10):
        code |= ((norm[:, 0] >> i) & 1) << (3 * i)
        code |= ((norm[:, 1] >> i) & 1) << (3 * i + 1)
        code |= ((norm[:, 2] >> i) & 1) << (3 * i + 2)
    assert len(torch.unique(code)) == n, "golden sample must have distinct Morton codes"
    out["morton_points"] = pts
    out["morton_codes"] = code.numpy()
    out["morton_adj"] = adj.astype(np.uint32)
    out["morton_offs"] = ip.astype(np.uint32)
    Infer._reorder_by_morton(obj)
    out["morton_new_points"] = obj.primal_points.numpy()
    out["morton_new_adj"] = obj.point_adjacency.numpy().astype(np.uint32)
    out["morton_new_offs"] = obj.point_adjacency_offsets.numpy().astype(np.uint32)

    # camera rays (reference convention)
    K = torch.tensor([[50.0, 0, 16.0], [0, 50.0, 12.0], [0, 0, 1.0]])
    T = torch.eye(4)
    T[:3, :3] = torch.tensor([[0.0, -1, 0], [0, 0, -1], [1, 0, 0]]).T
    T[:3, 3] = torch.tensor([3.0, 0.5, 0.25])
    out["cam_K"] = K.numpy()
    out["cam_T"] = T.numpy()
    out["cam_rays"] = vu.generate_camera_rays(K, T, 32, 24).numpy()
    np.savez_compressed(os.path.join(HERE, "layout_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "layout_golden.npz"))
    _foam_golden(root, vv)


def _foam_golden(root: str, vv):
    """Write .foam files with the reference exporter from a small seeded scene."""
    ds = types.ModuleType("vorotracing.datasets.datasets")
    ds.ColmapConfig = object
    sys.modules["vorotracing.datasets.datasets"] = ds
    sys.path.insert(0, os.path.join(root, "scripts"))
    import export_for_viewer as ex

    rng = np.random.default_rng(77)
    n, R = 40, 4
    pts = rng.uniform(-1, 1, (n, 3)).astype(np.float32)
    counts = rng.integers(3, 9, n)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
    adj = rng.integers(0, n, int(offs[-1]) + 32).astype(np.uint32)
    dens = rng.uniform(0, 2, (n, 1)).astype(np.float32)
    dif = rng.normal(size=(n, R * R * 4)).astype(np.float16)
    spe = rng.normal(size=(n, R * R * 4)).astype(np.float16)
    dif.reshape(n, -1, 4)[:, :, 3] = 0
    spe.reshape(n, -1, 4)[:, :, 3] = 0
    adj_diff = rng.normal(size=(adj.shape[0], 4)).astype(np.float16)
    poses = rng.normal(size=(3, 3, 4)).astype(np.float32)

    class Model:
        pass

    m = Model()
    m.primal_points = torch.from_numpy(pts)
    m.density = torch.from_numpy(dens)
    m.diffuse_fp16 = torch.from_numpy(dif)
    m.specular_fp16 = torch.from_numpy(spe)
    m.point_adjacency = torch.from_numpy(adj.astype(np.int64))
    m.point_adjacency_offsets = torch.from_numpy(offs.astype(np.int64))
    m.adjacent_diff = torch.from_numpy(adj_diff)
    cfg = vv.VoroTracingConfig(oct_map_res=R, spec_oct_map_res=R)
    aabb = (pts.min(0), pts.max(0))
    for version in (4, 3):
        ex.write_foam(os.path.join(HERE, f"scene_v{version}.foam"), m, cfg, poses, aabb[0],
                      aabb[1], 0.01, 1e-3, 512, include_specular=True, version=version)
    ex.write_foam(os.path.join(HERE, "scene_v4_nospec.foam"), m, cfg, poses, aabb[0], aabb[1],
                  0.01, 1e-3, 512, include_specular=False, version=4)
    np.savez_compressed(os.path.join(HERE, "foam_inputs.npz"), points=pts, density=dens,
                        diffuse=dif, specular=spe, adj=adj, offs=offs, adj_diff=adj_diff,
                        poses=poses)
    print("wrote .foam goldens")
    # reference checkpoint of a 16-site scene (R=4), written by the model itself
    cfg = vv.VoroTracingConfig(oct_map_res=4, spec_oct_map_res=4)
    k = 16
    model = vv.VoroTracing(cfg, torch.from_numpy(pts[:k]),
                           points_diffuse=torch.from_numpy(rng.normal(size=(k, 48)).astype(np.float32)),
                           points_specular=torch.from_numpy(rng.normal(size=(k, 48)).astype(np.float32)),
                           points_density=torch.from_numpy(rng.normal(size=(k, 1)).astype(np.float32)),
                           points_adjacency=torch.from_numpy(adj[:40].astype(np.int64) % k),
                           points_adjacency_offsets=torch.from_numpy(
                               np.minimum(np.arange(k + 1) * 2, 40).astype(np.int64)),
                           device=torch.device("cpu"))
    model.save_checkpoint(os.path.join(HERE, "checkpoint_ref.pt"))
    print("wrote checkpoint golden")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <path to the VoroTracing checkout>")
    main(sys.argv[1])
