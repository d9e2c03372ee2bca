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


def cpu_sample_rate(run, rays, budget_s=10.0):
    """Rays/s of a CPU oracle call ``run(sample_rays)`` on a strided sample of
    ``rays`` (N, 6) sized to about budget_s seconds; returns (rate, n, s)."""
    probe = rays[:: max(1, len(rays) // 1024)]
    t = time.perf_counter()
    run(probe)
    rate = len(probe) / max(time.perf_counter() - t, 1e-6)
    n = int(min(len(rays), max(1024, rate * budget_s)))
    sample = rays[:: max(1, len(rays) // n)][:n]
    t = time.perf_counter()
    run(sample)
    dt = time.perf_counter() - t
    return len(sample) / dt, len(sample), dt


def _cpu_line(rate, n, dt, total, unit_scale, unit, what):
    import oracle

    return {"value": rate / unit_scale, "unit": unit, "cores": oracle.max_threads(),
            "kind": "port",
            "sample": f"{n} of {total} rays (strided), {dt:.1f} s; {what}"}


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
    extra = {"fps": 64 * args.steps / (ms * 1e-3)}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        import oracle

        q8 = tuple(np.float32(v) for v in (scene.diff_scale, scene.diff_offset,
                                           scene.spec_scale, scene.spec_offset))
        h = lambda x: x.detach().cpu().numpy()
        S = oracle.Scene(h(scene.primal_points), h(scene.point_adjacency),
                         h(scene.point_adjacency_offsets), h(scene.density), h(scene.diffuse_q8),
                         h(scene.specular_q8), oracle.ATTR_U8, q8=q8)
        r0 = views[0].reshape(-1, 6).cpu().numpy()
        st0 = int(starts[0].reshape(-1)[0])
        thr = oracle.max_threads()
        rate, n, dt = cpu_sample_rate(
            lambda r: oracle.trace_infer(S, r, np.full(len(r), st0, np.uint32), wt=WT,
                                         skip=SKIP, threads=thr), r0)
        extra["cpu_baseline"] = _cpu_line(rate, n, dt, len(r0), 1e6, "Mrays/s",
                                          "q8 inference of view 0 by the CPU restatement")
    if rank == 0:
        rays = 64 * W * H * args.steps
        _line(args, ws, "Mrays/s q8 forward render, 64 views 1296x840, 1M-site scene (C3)",
              rays / (ms * 1e-3) / 1e6, "Mrays/s", ms, clocks,
              {"workload": "C3: C2 scene with q8 textures (global scale/offset per map), 64 "
                           "orbit views (radius 3, elevation 15 deg), view-sharded",
               "views_per_step": 64, "parallelism": f"views round-robin over {ws} GPU(s)",
               "l2": "flushed between timed steps (256 MB write)"},
              "strong", "f32", extra)


def c4_setup(ws, rank, dev, n_sites=None, attrs_on_device=False, allreduce="peer"):
    """The C4 training workload of this rank: scene tensors, this rank's
    1552x1040 camera (orbit view = rank) in 4x8 tile order, broadcast start
    cell, seeded target, gradient bucket and path record.

    attrs_on_device: draw density / texture logits with torch's generator on
    the GPU (same distributions as scene.make_scene, other values) instead of
    numpy on the host -- seconds instead of a minute per rank for the 4.6 GB
    of texels, used by the training leg of ``bench.py --gpus N``."""
    from vorotracing_b200.cuda import NNBVH
    from vorotracing_b200.cuda import _ops as ops_

    c = sc.CONFIGS["C4"]
    if attrs_on_device:
        n = n_sites or c["n"]
        pts = sc.make_sites(n, c["seed"], c["plane"])
        t = {"points": torch.from_numpy(pts).to(dev)}
        adj, offs, _ = ops_.build_voronoi_adjacency(t["points"], chunk_padding=sc.CSR_PAD)
        t["adj"], t["offs"] = adj, offs
        g = torch.Generator(device=dev).manual_seed(c["seed"] + 1000)
        cols = 3 * c["res"] * c["res"]
        t["density"] = torch.nn.functional.softplus(
            torch.randn((n, 1), generator=g, device=dev))
        t["diffuse"] = torch.rand((n, cols), generator=g, device=dev)
        t["specular"] = torch.rand((n, cols), generator=g, device=dev) - 0.5
    else:
        s = bench.load_scene(rank, ws, "C4", adjacency="gpu", n=n_sites)
        t = _scene_tensors(s, dev)
    W, H = c["W"], c["H"]
    rays = torch.from_numpy(sc.pinhole_rays(sc.intrinsics(W, H), sc.orbit_pose(rank, 64), W,
                                            H)).to(dev)
    bvh = NNBVH()
    bvh.build(t["points"])
    st0 = bvh.query(t["points"], rays[0, 0, :3].reshape(1, 3))
    start = st0.expand(H * W).contiguous().view(torch.uint32)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    target = torch.rand((H, W, 3), generator=gen, device=dev)
    # Batch order is free in training (the reference samples patch-coherent
    # batches, vorotracing/datasets/datasets.py:238-241): rays and target go
    # in 4x8 tile order so that a warp traces neighbouring pixels.
    perm = ops_.tile_perm(H, W, device=dev).long()
    rays = rays.reshape(-1, 6)[perm].contiguous()
    target = target.reshape(-1, 3)[perm].contiguous()
    n = t["points"].size(0)
    bucket = GradBucket(n, t["diffuse"].size(1), dev)
    nr = H * W
    # the forward records each ray's first 384 steps (cell + segment colour);
    # the backward replays them without scanning faces or re-reading texels
    # (6 KB per ray; at 256 steps 0.4 % of C4's rays overflowed and were
    # walked again, 36.75 vs 36.13 ms per step)
    path = ops_.PathRecord(nr, 384, dev)
    w = dict(t=t, rays=rays, start=start, target=target, bucket=bucket, path=path, nr=nr, n=n,
             reducer=None, allreduce="nccl" if ws == 1 else allreduce)
    if ws > 1 and allreduce == "peer":
        from vorotracing_b200.shard import PeerGradReducer

        # every rank takes the same branch: the setup's outcome is agreed on
        # through the process group before anything depends on it
        red, why = None, None
        try:
            red = PeerGradReducer(bucket, c["res"])
        except RuntimeError as e:
            why = f"peer mapping failed: {e}"
        ok = torch.tensor([0 if red is None else 1], dtype=torch.int32, device=dev)
        torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
        if int(ok.item()) == 1:
            w["reducer"] = red
            chk = _check_peer_reduce(w)
            w["peer_check"] = chk
            if not chk["rel"] <= 1e-4:  # agreed: every rank computed the same buckets
                why = f"peer result differs from NCCL's (rel {chk['rel']:.3g})"
        elif why is None:
            why = "peer mapping failed on another rank"
        if why is not None:
            if red is not None:
                red.close()
            w["reducer"], w["allreduce"] = None, "nccl"
            w["peer_fallback"] = why
    return w


def _check_peer_reduce(w):
    """One step's gradients reduced both ways, the fused peer kernel and
    NCCL's all-reduce of the compacted bucket: the largest difference
    relative to the gradient's scale (summation orders differ)."""
    c4_step_fn(w, reduce=False)()
    red = w["reducer"]
    red.reduce_()
    peer = w["bucket"].flat.clone()
    w_n = dict(w, reducer=None, allreduce="nccl")
    c4_step_fn(w_n)()
    torch.cuda.synchronize()
    ref = w["bucket"].flat
    scale = float(ref.abs().max())
    diff = float((peer - ref).abs().max())
    del peer
    return {"max_abs_diff": diff, "scale": scale, "rel": diff / scale if scale else 0.0}


def c4_step_fn(w, ar_events=None, reduce=True):
    """One training step: face pack + forward (recording paths) + MSE
    gradient + backward (replaying them) into the flat bucket + the
    all-reduce of the bucket: NCCL's, or (w["reducer"]) the fused
    compaction + reduction over peer memory.  ar_events: a list that
    receives an (start, end) CUDA event pair around the reduction of every
    call; reduce=False stops after the backward."""
    from vorotracing_b200.cuda import _ops

    t, rays, start, target = w["t"], w["rays"], w["start"], w["target"]
    bucket, path, nr = w["bucket"], w["path"], w["nr"]
    red = w.get("reducer")
    bw = dict(workspace=red.workspace, keep_workspace=True) if red is not None else {}

    def do_reduce():
        if red is not None:
            red.reduce_()
        else:
            bucket.allreduce_()

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
                                   grads=bucket.views(), path=path, accumulate=False, **bw)
        if not reduce:
            return
        if ar_events is not None:
            e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            e[0].record()
            do_reduce()
            e[1].record()
            ar_events.append(e)
        else:
            do_reduce()

    return step


C4_METRIC = "training rays/s, fwd+bwd+grad all-reduce, 3M-site scene, 1552x1040 per GPU (C4)"
C4_WORKLOAD = ("C4: 3M-site fp32 scene, R=8, one 1552x1040 camera per GPU vs a seeded U(0,1) "
               "target, MSE; step = face pack + fwd (recording each ray's first 384 steps: "
               "cell + colour) + bwd (replaying them) + NCCL all-reduce of the flat fp32 "
               "gradient bucket; optimizer excluded")


def c4_measure(args, ws, dev, w, steps, warmup):
    """Times `steps` C4 steps (CUDA events, L2 flushed, max over ranks);
    returns the step time, the all-reduce share and NCCL's bus bandwidth."""
    ar = []
    step = c4_step_fn(w, ar)

    class A:
        pass

    a = A()
    a.steps, a.warmup = steps, warmup
    ms, clocks = Timer(a, dev).run(step, ws)
    timed = ar[-steps:]
    ar_ms = sum(x.elapsed_time(y) for x, y in timed) / steps
    v = torch.tensor([ar_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
    ar_ms = float(v.item())
    nbytes = w["bucket"].nbytes
    busbw = (2.0 * (ws - 1) / ws * nbytes / (ar_ms * 1e-3) / 1e9) if ws > 1 and ar_ms > 0 else None
    return dict(ms_total=ms, ms_per_step=ms / steps, clocks=clocks, allreduce_ms=ar_ms,
                allreduce_bus_gbs=busbw, bucket_bytes=nbytes, allreduce=w["allreduce"],
                peer_check=w.get("peer_check"), peer_fallback=w.get("peer_fallback"),
                rays_per_s=w["nr"] * ws * steps / (ms * 1e-3))


def run_c4(args, ws, rank, dev):
    w = c4_setup(ws, rank, dev, n_sites=args.sites, allreduce=args.allreduce)
    if args.profile:
        step = c4_step_fn(w)
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        return
    r = c4_measure(args, ws, dev, w, args.steps, args.warmup)
    extra = {"allreduce_ms_per_step": r["allreduce_ms"],
             "allreduce_bus_gbs": r["allreduce_bus_gbs"], "allreduce": r["allreduce"],
             "peer_check": r["peer_check"], "peer_fallback": r["peer_fallback"]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        import oracle

        h = lambda x: x.detach().cpu().numpy()
        t = w["t"]
        S = oracle.Scene(h(t["points"]), h(t["adj"]), h(t["offs"]), h(t["density"]),
                         h(t["diffuse"]), h(t["specular"]), oracle.ATTR_F32)
        rays_h = h(w["rays"])
        st0 = int(w["start"][0])
        thr = oracle.max_threads()

        def train(rr):
            st = np.full(len(rr), st0, np.uint32)
            f = oracle.trace_fwd(S, rr, st, wt=WT, threads=thr)
            g = np.zeros_like(f["rgba"])
            g[:, :3] = (2.0 / (len(rr) * 3)) * (f["rgba"][:, :3] - 0.5)
            oracle.trace_bwd(S, rr, st, f["rgba"], g, W=f["W"], S=f["S"], t_far=f["t_far"],
                             distortion=f["distortion"], wt=WT, threads=thr)

        rate, n, dt = cpu_sample_rate(train, rays_h)
        extra["cpu_baseline"] = _cpu_line(rate, n, dt, len(rays_h), 1.0, "rays/s",
                                          "training forward + backward by the CPU restatement "
                                          "(no all-reduce)")
    if rank == 0:
        _line(args, ws, C4_METRIC, r["rays_per_s"], "rays/s", r["ms_total"], r["clocks"],
              {"workload": C4_WORKLOAD, "sites": w["n"], "rays_per_step_per_gpu": w["nr"],
               "grad_bucket_bytes": r["bucket_bytes"],
               "parallelism": f"data-parallel x{ws} (rays), scene replicated",
               "l2": "flushed between timed steps (256 MB write)"},
              "weak", "f32", extra)


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
    extra = {}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        import oracle

        h = lambda x: x.detach().cpu().numpy()
        S = oracle.Scene(h(scene.primal_points), h(scene.point_adjacency),
                         h(scene.point_adjacency_offsets), h(scene.density),
                         h(scene.diffuse_fp16), h(scene.specular_fp16), oracle.ATTR_F16X4)
        allr = np.concatenate([h(f).reshape(-1, 6) for f in frames])
        pts = h(scene.primal_points)
        thr = oracle.max_threads()

        from scipy.spatial import cKDTree

        tree = cKDTree(pts.astype(np.float64))

        def infer(rr):
            # start cells: scipy's k-d tree (built once, outside the timing)
            st = tree.query(rr[:, :3].astype(np.float64), workers=thr)[1].astype(np.uint32)
            oracle.trace_infer(S, rr, st, wt=WT, skip=SKIP, threads=thr)

        rate, n, dt = cpu_sample_rate(infer, allr)
        extra["cpu_baseline"] = _cpu_line(rate, n, dt, len(allr), 1e6, "Mrays/s",
                                          "per-ray start cell (scipy cKDTree) + fp16 inference "
                                          "by the CPU restatement, all three cameras")
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
              "strong", "f32", extra)


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
