"""Benchmark configurations other than the headline C2 (``bench.py --config``).

  C3  1M-site scene, q8 textures (one global scale/offset per map), 64 orbit
      views at 1296x840 sharded by view over the ranks (strong scaling:
      the 64 views are the fixed total).  Metric: Mrays/s, frames/s.
  C4  training step on a 3M-site fp32 scene: one 1552x1040 camera per rank
      (orbit view = rank, rays in 4x8 tile order) against a seeded U(0,1)
      target image; a step is
      packed-face rebuild + forward + MSE gradient + backward + NCCL
      all-reduce of the flat fp32 gradient bucket (optimizer excluded).
      Metric: training rays/s (weak scaling).
  C5  4M-site fp16 scene, 1920x1080: an equidistant fisheye (190 deg), a
      rolling-shutter pinhole (30 ms readout, 1 m/s) and a thin-lens pinhole
      (aperture radius 0.02, focus 3, 4 stratified samples per pixel); every
      ray gets its own start cell from the BVH; pixel rows are dealt to the
      ranks in 4-row bands (strong scaling).  Metric: Mrays/s.

Scenes: C2/C3 use scipy/Qhull adjacency (as the parity tests do); the 3M- and
4M-site C4/C5 scenes are built with the GPU Voronoi builder (seconds instead
of minutes of host time).

Timing follows bench.py: CUDA events per step on the launching stream, L2
flushed between steps, max over ranks, nvidia-smi clocks sampled meanwhile.
"""
from __future__ import annotations

import json
import os
import time

import numpy as np
import torch

import bench
from vorotracing_b200 import scene as sc
from vorotracing_b200.shard import GradBucket, row_band_shard, view_shard

WT, SKIP = 0.01, 1e-3


class Timer:
    def __init__(self, args, dev):
        self.args = args
        self.dev = dev
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def run(self, step, ws):
        """Warm up, then time args.steps calls of step(); returns (ms total, clocks)."""
        for _ in range(max(self.args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        sampler = bench.ClockSampler(self.dev.index)
        sampler.start()
        time.sleep(0.3)
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(self.args.steps)]
        for k in range(self.args.steps):
            self.flush.fill_(k & 0xFF)
            ev[k][0].record()
            step()
            ev[k][1].record()
        torch.cuda.synchronize()
        if ws > 1:
            torch.distributed.barrier()
        clocks = sampler.stop()
        ms = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64,
                          device=self.dev)
        if ws > 1:
            torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
        return float(ms.item()), clocks


def _line(args, ws, metric, value, unit, ms_total, clocks, config, scaling, dtype, extra=None):
    out = {"metric": metric, "value": value, "unit": unit, "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
           "scaling": scaling, "vs_baseline": None, "dtype": dtype, "data": "synthetic",
           "config": config, "clocks": clocks}
    out.update(extra or {})
    print(json.dumps(out), flush=True)


def _scene_tensors(s, dev):
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return {k: d(s[k]) for k in ("points", "density", "adj", "offs", "diffuse", "specular")}


def run_c3(args, ws, rank, dev):
    from vorotracing_b200.cameras import Camera
    from vorotracing_b200.render import InferScene

    s = bench.load_scene(rank, ws, "C3")
    t = _scene_tensors(s, dev)
    scene = InferScene(t["points"], t["density"], t["adj"], t["offs"], t["diffuse"],
                       t["specular"], quantize="q8", sort_morton=True)
    del t
    W, H = sc.CONFIGS["C3"]["W"], sc.CONFIGS["C3"]["H"]
    K = sc.intrinsics(W, H)
    mine = view_shard(64, rank, ws)
    views = [Camera.pinhole(K, sc.orbit_pose(v, 64), W, H).rays(dev) for v in mine]
    starts = [scene.get_starting_point(r) for r in views]

    def step():
        for r, st in zip(views, starts):
            scene.render(r, start_point=st, weight_threshold=WT, cell_skip_threshold=SKIP)

    ms, clocks = Timer(args, dev).run(step, ws)
    if rank == 0:
        rays = 64 * W * H * args.steps
        _line(args, ws, "Mrays/s q8 forward render, 64 views 1296x840, 1M-site scene (C3)",
              rays / (ms * 1e-3) / 1e6, "Mrays/s", ms, clocks,
              {"workload": "C3: C2 scene with q8 textures (global scale/offset per map), 64 "
                           "orbit views (radius 3, elevation 15 deg), view-sharded",
               "views_per_step": 64, "parallelism": f"views round-robin over {ws} GPU(s)",
               "l2": "flushed between timed steps (256 MB write)"},
              "strong", "f32", {"fps": 64 * args.steps / (ms * 1e-3)})


def run_c4(args, ws, rank, dev):
    from vorotracing_b200.cuda import _ops

    s = bench.load_scene(rank, ws, "C4", adjacency="gpu", n=args.sites)
    t = _scene_tensors(s, dev)
    W, H = sc.CONFIGS["C4"]["W"], sc.CONFIGS["C4"]["H"]
    rays = torch.from_numpy(sc.pinhole_rays(sc.intrinsics(W, H), sc.orbit_pose(rank, 64), W, H)).to(dev)
    from vorotracing_b200.cuda import NNBVH

    bvh = NNBVH()
    bvh.build(t["points"])
    st0 = bvh.query(t["points"], rays[0, 0, :3].reshape(1, 3))
    start = st0.expand(H * W).contiguous().view(torch.uint32)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    target = torch.rand((H, W, 3), generator=gen, device=dev)
    # Batch order is free in training (the reference samples patch-coherent
    # batches, vorotracing/datasets/datasets.py:238-241): rays and target go
    # in 4x8 tile order so that a warp traces neighbouring pixels.
    from vorotracing_b200.cuda import _ops as ops_

    perm = ops_.tile_perm(H, W, device=dev).long()
    rays = rays.reshape(-1, 6)[perm].contiguous()
    target = target.reshape(-1, 3)[perm].contiguous()
    n = t["points"].size(0)
    bucket = GradBucket(n, t["diffuse"].size(1), dev)
    nr = H * W
    # the forward records each ray's first 256 steps (cell + segment colour);
    # the backward replays them without scanning faces or re-reading texels
    # (4 KB per ray)
    path = ops_.PathRecord(nr, 256, dev)

    def step():
        faces = _ops.prefetch_faces(t["points"], t["adj"], t["offs"])
        rgba, _, _, _, _, dist_, Wt, St, tfar = _ops.trace_vorotracing_fwd(
            t["points"], t["diffuse"], t["specular"], t["density"], t["adj"], t["offs"], rays,
            start, None, WT, 1024, False, faces=faces, path=path)
        g = torch.zeros_like(rgba)
        g[:, :3] = (2.0 / (nr * 3)) * (rgba[:, :3] - target)
        _ops.trace_vorotracing_bwd(t["points"], t["diffuse"], t["specular"], t["density"],
                                   t["adj"], t["offs"], rays, start, rgba, g, None, None, None,
                                   None, 0.0, dist_, None, Wt, St, tfar, WT, 1024, faces=faces,
                                   grads=bucket.views(), path=path, accumulate=False)
        bucket.allreduce_()

    if args.profile:
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        return
    ms, clocks = Timer(args, dev).run(step, ws)
    if rank == 0:
        rays_total = nr * ws * args.steps
        _line(args, ws, "training rays/s, fwd+bwd+grad all-reduce, 3M-site scene, 1552x1040 per GPU (C4)",
              rays_total / (ms * 1e-3), "rays/s", ms, clocks,
              {"workload": "C4: 3M-site fp32 scene, R=8, one 1552x1040 camera per GPU vs a "
                           "seeded U(0,1) target, MSE; step = face pack + fwd (recording each "
                           "ray's first 256 steps: cell + colour) + bwd (replaying them) + NCCL "
                           "all-reduce of the flat fp32 gradient bucket; optimizer excluded",
               "sites": n, "rays_per_step_per_gpu": nr,
               "grad_bucket_bytes": bucket.nbytes,
               "parallelism": f"data-parallel x{ws} (rays), scene replicated",
               "l2": "flushed between timed steps (256 MB write)"},
              "weak", "f32")


def run_c5(args, ws, rank, dev):
    from vorotracing_b200.cameras import FISHEYE, ROLLING, THIN_LENS, Camera
    from vorotracing_b200.render import InferScene

    s = bench.load_scene(rank, ws, "C5", adjacency="gpu")
    t = _scene_tensors(s, dev)
    scene = InferScene(t["points"], t["density"], t["adj"], t["offs"], t["diffuse"],
                       t["specular"], quantize="fp16", sort_morton=True)
    del t
    W, H = sc.CONFIGS["C5"]["W"], sc.CONFIGS["C5"]["H"]
    K = sc.intrinsics(W, H)
    T = sc.orbit_pose(0, 64)
    fe = Camera.fisheye(T, W, H, 190.0)
    rs = Camera.pinhole(K, T, W, H)
    rs.model, rs.rs_duration, rs.velocity = ROLLING, 0.03, tuple(T[:3, 0])  # 1 m/s sideways
    tl = Camera.pinhole(K, T, W, H)
    tl.model, tl.spp, tl.lens_radius, tl.focus_distance, tl.seed = THIN_LENS, 4, 0.02, 3.0, 5
    rows = torch.from_numpy(row_band_shard(H, rank, ws)).to(dev)
    frames = []
    for cam in (fe, rs, tl):
        r = cam.rays(dev).index_select(0, rows).contiguous()
        # image-shaped (rows, W * spp, 6): the render then traces in 4x8 warp
        # tiles (the lens samples of a pixel are adjacent columns)
        frames.append(r.reshape(r.size(0), -1, 6))
    nr = sum(f.numel() // 6 for f in frames)

    def step():
        for r in frames:
            scene.render(r, weight_threshold=WT, cell_skip_threshold=SKIP, per_ray_start=True)

    ms, clocks = Timer(args, dev).run(step, ws)
    tot = torch.tensor([nr], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(tot)
    if rank == 0:
        rays_total = float(tot.item()) * args.steps
        _line(args, ws, "Mrays/s non-pinhole forward render, 4M-site scene, 1920x1080 fisheye + rolling shutter + thin lens x4 (C5)",
              rays_total / (ms * 1e-3) / 1e6, "Mrays/s", ms, clocks,
              {"workload": "C5: 4M-site fp16 scene; equidistant fisheye 190 deg, rolling "
                           "shutter (30 ms, 1 m/s), thin lens (r 0.02, focus 3, 4 spp); per-ray "
                           "BVH start cells inside the step; 4-row bands over the GPUs",
               "rays_per_step": int(tot.item()),
               "parallelism": f"4-row bands round-robin over {ws} GPU(s)",
               "l2": "flushed between timed steps (256 MB write)"},
              "strong", "f32")


def run(args):
    ws, rank, local = bench._dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    try:
        {"C3": run_c3, "C4": run_c4, "C5": run_c5}[args.config](args, ws, rank, dev)
    finally:
        if ws > 1:
            torch.distributed.destroy_process_group()
