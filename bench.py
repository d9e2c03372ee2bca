"""Benchmark of the Voronoi ray-traversal hot path (forward render, config C2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("C2"): a seeded synthetic 1M-site Voronoi scene
(70 % noisy sphere + ground plane, 30 % uniform), fp16 8x8 octahedral
textures, Morton-sorted cells, 4x8 warp tiles, one 1296x840 pinhole view per
GPU (rank r renders orbit view r), weight_threshold 0.01, cell_skip 1e-3.
A step = start-cell lookup + full-frame traversal render.  Scene arrays are
resident in HBM before timing; L2 is flushed (256 MB write) between timed
steps.  `e2e` renders through InferScene.render_host from page-locked host
rays to page-locked host rgba, the bus transfers inside the timed region (by
default the trace kernel reads and writes host memory directly).

Multi-GPU: one process per GPU (torchrun), the scene is replicated, views are
independent (weak scaling, no collective on the data path); time = max over
ranks.  --impl reference times the CPU restatement of the reference's
algorithm (the reference's own CUDA extension cannot be built: its Eigen
and cuBQL submodules are empty) on all host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Mrays/s forward render, 1296x840 view of a 1M-site Voronoi scene (C2)"
WORKLOAD = ("C2: 1M-site seeded synthetic Voronoi scene (sphere+plane+uniform), fp16 8x8 "
            "octahedral textures, fp32 density, Morton-sorted, 4x8 warp tiles, one 1296x840 "
            "pinhole view per GPU, weight_threshold 0.01, cell_skip_threshold 1e-3")
WT, SKIP = 0.01, 1e-3


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def load_scene(rank: int, ws: int, name: str = "C2", adjacency: str = "qhull", n=None):
    """Scene arrays of a configuration (``n`` overrides the site count, for
    small profiling captures); rank 0 builds the adjacency cache first."""
    from vorotracing_b200 import scene as sc

    if ws > 1:
        import torch.distributed as dist

        if rank == 0:
            sc.config_scene(name, n=n, adjacency=adjacency)
        dist.barrier()
    return sc.config_scene(name, n=n, adjacency=adjacency)


def compulsory_bytes(scene, rays, start, dbg_ops):
    """Bytes the frame must move at least once: every visited cell's face rows
    (16 B each), site (12 B) and density (4 B) and CSR offsets of the start
    cell, 64 B of texels per textured cell, plus rays (24 B), start (4 B), ray
    permutation (4 B) and rgba (8 B) per ray."""
    import torch

    dbg = {"visited": True}
    scene.render(rays, start_point=start, weight_threshold=WT, cell_skip_threshold=SKIP,
                 debug=dbg)
    torch.cuda.synchronize()
    offs = scene.point_adjacency_offsets.to(torch.int64)
    deg = (offs[1:] - offs[:-1]).to(torch.float64)
    vis = dbg["visited"].to(torch.float64)
    tex = dbg["textured"].to(torch.float64)
    nr = rays.numel() // 6
    cells = float((vis * (16.0 * deg + 16.0)).sum()) + float(tex.sum()) * 64.0 + 8.0
    per_ray_io = 24.0 + 4.0 + 4.0 + 8.0
    st = dbg["stats"].to(torch.float64).mean(0).cpu().numpy()
    # bytes each ray reads through L1/L2 (re-reads included), this layout
    cached = per_ray_io + st[0] * 16.0 + st[1] * 16.0 + st[3] * 64.0
    return cells + per_ray_io * nr, dict(steps=st[0], faces=st[1], segments=st[2],
                                          textured=st[3], bytes_per_ray_l1l2=cached,
                                          visited_cells=int(vis.sum()),
                                          textured_cells=int(tex.sum()))


def algorithmic_bytes_per_ray(stats, tex_bytes: float) -> float:
    """Bytes a ray touches by the reference's accounting: 40 B of ray I/O
    (ray 24, start 4, permutation 4, rgba 8) plus, per visited cell, 28 B
    (CSR offsets 8, winning neighbour id 4, next site 12, density 4), 8 B per
    face tested (a half4 neighbour difference) and the cell's texels when it
    is textured (64 B fp16, 24 B q8, 96 B fp32)."""
    return (40.0 + 28.0 * float(stats["steps"]) + 8.0 * float(stats["faces"])
            + tex_bytes * float(stats["textured"]))


def cpu_oracle_rate(s, rays_np, start_idx, budget_s=15.0, threads=0, max_rays=None):
    """Rays/s of the CPU restatement on a strided sample sized to ~budget_s."""
    import oracle
    from oracle import pad_f16x4

    res = s["res"]
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"],
                     pad_f16x4(s["diffuse"], res), pad_f16x4(s["specular"], res),
                     oracle.ATTR_F16X4)
    flat = rays_np.reshape(-1, 6)
    probe = flat[:: max(1, len(flat) // 4096)]
    t = time.perf_counter()
    oracle.trace_infer(S, probe, np.full(len(probe), start_idx, np.uint32), wt=WT, skip=SKIP,
                       threads=threads)
    rate = len(probe) / (time.perf_counter() - t)
    n = int(min(len(flat), max(4096, rate * budget_s)))
    if max_rays:
        n = min(n, max_rays)
    sample = flat[:: max(1, len(flat) // n)][:n]
    t = time.perf_counter()
    oracle.trace_infer(S, sample, np.full(len(sample), start_idx, np.uint32), wt=WT, skip=SKIP,
                       threads=threads)
    dt = time.perf_counter() - t
    return len(sample) / dt, len(sample), dt, S


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    import oracle
    from vorotracing_b200 import scene as sc

    s = sc.config_scene("C2")
    rays = sc.config_rays("C2", view=0)
    st = int(oracle.nn_query(s["points"], rays.reshape(-1, 6)[:1, :3])[0])
    threads = oracle.max_threads()
    rate, n, dt, S = cpu_oracle_rate(s, rays, st, budget_s=1.0, threads=threads)
    flat = rays.reshape(-1, 6)
    sample = flat[:: max(1, len(flat) // n)][:n]
    start = np.full(len(sample), st, np.uint32)
    for _ in range(args.warmup):
        oracle.trace_infer(S, sample, start, wt=WT, skip=SKIP, threads=threads)
    t = time.perf_counter()
    for _ in range(args.steps):
        oracle.trace_infer(S, sample, start, wt=WT, skip=SKIP, threads=threads)
    dt = time.perf_counter() - t
    v = len(sample) * args.steps / dt / 1e6
    full = flat.shape[0]
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "Mrays/s",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": dt / args.steps * 1e3, "fps": v * 1e6 / full,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": {"workload": WORKLOAD},
           "cpu_baseline": {"value": v, "unit": "Mrays/s", "cores": threads, "kind": "port",
                            "sample": f"{len(sample)} rays per step, strided over view 0 "
                                      f"({full} rays)"},
           "e2e": {"value": v, "unit": "Mrays/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0},
           "note": "CPU restatement of the reference traversal (oracle/vto_oracle.c), OpenMP "
                   "over rays; the reference CUDA extension cannot be built here"}
    print(json.dumps(out), flush=True)


def training_leg(ws, rank, dev, steps, allreduce="peer"):
    """C4 training rays/s at this run's GPU count (every rank takes part):
    one 1552x1040 camera per GPU on the 3M-site scene, fwd + bwd + the
    gradient all-reduce of the 4.66 GB bucket per step (weak scaling).  At
    N > 1 with allreduce="peer" both reductions are timed, the fused
    compaction + all-reduce over peer memory and the compaction + NCCL
    all-reduce, and the faster one is reported (both timings are listed)."""
    import torch

    import bench_configs as bc

    w = bc.c4_setup(ws, rank, dev, attrs_on_device=True, allreduce=allreduce)
    r = bc.c4_measure(None, ws, dev, w, steps, 3)
    timings = {r["allreduce"]: r["ms_per_step"]}
    if ws > 1 and w.get("reducer") is not None:
        alt = bc.c4_measure(None, ws, dev, dict(w, reducer=None, allreduce="nccl"), steps, 3)
        timings["nccl"] = alt["ms_per_step"]
        if alt["ms_per_step"] < r["ms_per_step"]:
            alt["peer_check"] = r["peer_check"]
            r = alt
    res = {"metric": bc.C4_METRIC, "value": r["rays_per_s"], "unit": "rays/s",
           "steps": steps, "warmup": 3, "ms_per_step": r["ms_per_step"],
           "allreduce_ms_per_step": r["allreduce_ms"],
           "allreduce_bus_gbs": r["allreduce_bus_gbs"], "grad_bucket_bytes": r["bucket_bytes"],
           "allreduce": r["allreduce"], "ms_per_step_by_allreduce": timings,
           "peer_check": r["peer_check"], "peer_fallback": r["peer_fallback"],
           "scaling": "weak", "clocks": r["clocks"],
           "config": {"workload": bc.C4_WORKLOAD, "sites": w["n"],
                      "rays_per_step_per_gpu": w["nr"],
                      "attributes": "drawn on the device (torch generator, same distributions "
                                    "as the seeded numpy scene)",
                      "l2": "flushed between timed steps (256 MB write)"}}
    if w.get("reducer") is not None:
        w["reducer"].close()
    del w
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"],
                    help="C4 gradient reduction at N>1: the fused compaction + all-reduce over "
                         "peer memory, or the compaction then NCCL's all-reduce")
    ap.add_argument("--no-train-leg", action="store_true",
                    help="skip the C4 training leg of the C2 line")
    ap.add_argument("--transfer", default="zero_copy", choices=["zero_copy", "bands"],
                    help="e2e host I/O: the kernel reads/writes page-locked host memory "
                         "directly, or banded copies overlapped with the trace")
    ap.add_argument("--bands", type=int, default=4, help="row bands of --transfer bands")
    ap.add_argument("--config", default="C2", choices=["C2", "C3", "C4", "C5"],
                    help="C2 (default, the headline) or another benchmark configuration")
    ap.add_argument("--profile", action="store_true",
                    help="a few untimed steps only (for ncu captures)")
    ap.add_argument("--sites", type=int, default=None,
                    help="override the configuration's site count (small ncu captures with "
                         "--profile; never for a reported number)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.config != "C2":
        import bench_configs

        return bench_configs.run(args)

    import torch

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.render import InferScene

    if args.sites is not None and not args.profile:
        raise SystemExit("--sites is for --profile captures only")
    s = (load_scene(rank, ws) if args.sites is None
         else load_scene(rank, ws, adjacency="gpu", n=args.sites))
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    scene = InferScene(d(s["points"]), d(s["density"]), d(s["adj"]), d(s["offs"]),
                       d(s["diffuse"]), d(s["specular"]), quantize="fp16", sort_morton=True)
    rays_np = sc.config_rays("C2", view=rank)
    H, W = rays_np.shape[:2]
    nr = H * W
    rays = d(rays_np)
    rays_host = torch.from_numpy(rays_np).pin_memory()
    out_host = torch.empty((H, W, 4), dtype=torch.float16, pin_memory=True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def render():
        return scene.render(rays, weight_threshold=WT, cell_skip_threshold=SKIP)

    if args.profile:
        for _ in range(3):
            render()
        torch.cuda.synchronize()
        return

    for _ in range(max(args.warmup, 3)):
        render()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for k in range(args.steps):
        flush.fill_(k & 0xff)
        e0, e1, e2 = ev[k]
        e0.record()
        start = scene.get_starting_point(rays)
        e1.record()
        scene.render(rays, start_point=start, weight_threshold=WT, cell_skip_threshold=SKIP)
        e2.record()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    trace_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps

    # end to end: pinned host rays -> device, render, rgba -> pinned host
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for _ in range(2):
        scene.render_host(rays_host, out_host, transfer=args.transfer, bands=args.bands,
                          weight_threshold=WT,
                          cell_skip_threshold=SKIP)
    for k in range(args.steps):
        flush.fill_(k & 0xff)
        a, b = e2e_ev[k]
        a.record()
        scene.render_host(rays_host, out_host, transfer=args.transfer, bands=args.bands,
                          sync=False,
                          weight_threshold=WT, cell_skip_threshold=SKIP)
        b.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev)
    n_bands = 1
    if args.transfer == "bands" and args.bands > 1:
        n_bands = len(range(0, H, -(-H // (args.bands * 4)) * 4))

    t = torch.tensor([step_ms, e2e_ms, trace_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    step_ms, e2e_ms, trace_ms = (float(x) for x in t.cpu())
    if rank != 0:
        if not args.no_train_leg:
            training_leg(ws, rank, dev, min(args.steps, 10), args.allreduce)
        torch.distributed.destroy_process_group()
        return

    total_rays = nr * args.steps * ws
    value = total_rays / (step_ms * 1e-3) / 1e6
    e2e_value = total_rays / (e2e_ms * 1e-3) / 1e6
    comp, stats = compulsory_bytes(scene, rays, scene.get_starting_point(rays), None)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        hbm = json.load(open(peaks_path))["hbm_gbs"]
        peak_src = "measured"
    else:
        hbm, peak_src = 6650.0, "fallback"
    # the contract's algorithmic bytes (the reference's per-cell reads):
    # B_ray = 40 + sum over cells (28 + 8 * faces scanned + 64 if textured)
    b_ray = algorithmic_bytes_per_ray(stats, 64.0)
    alg = b_ray * nr
    achieved = alg / (trace_ms * 1e-3) / 1e9
    comp_achieved = comp / (trace_ms * 1e-3) / 1e9
    traffic = None
    warp_inst = None
    prof = os.path.join(ROOT, "profiles", "trace_infer_f16_c2.json")
    if os.path.exists(prof):
        pj = json.load(open(prof))
        traffic = pj.get("dram_bytes_per_launch")
        warp_inst = pj.get("warp_instructions_per_launch")
    issue = None
    if warp_inst:
        # the kernel is instruction-issue bound: one warp instruction per cycle
        # per SM sub-partition (4 per SM, 148 SMs) at the sampled SM clock
        sm_hz = float(clocks.get("sm_mhz") or 1965.0) * 1e6
        peak_issue = 148 * 4 * sm_hz
        got_issue = warp_inst / (trace_ms * 1e-3)
        issue = {"achieved": got_issue, "peak": peak_issue, "unit": "warp instructions/s",
                 "frac": got_issue / peak_issue, "warp_instructions_per_launch": warp_inst,
                 "source": "ncu smsp__inst_executed.sum of the same kernel (profiles/)"}
    out = {
        "metric": METRIC, "value": value, "unit": "Mrays/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms / args.steps,
        "fps": 1000.0 / (step_ms / args.steps), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sites": int(s["points"].shape[0]),
                   "rays_per_step_per_gpu": nr, "l2": "flushed between timed steps (256 MB write)",
                   "parallelism": f"view-sharded x{ws}, scene replicated"},
        "e2e": {"value": e2e_value, "unit": "Mrays/s", "h2d_bytes_per_step": nr * 24,
                "d2h_bytes_per_step": nr * 8, "transfer": args.transfer, "bands": n_bands,
                "how": ("InferScene.render_host: the trace kernel reads the rays from and "
                        "writes the f16 rgba to page-locked host memory over the bus "
                        "(zero-copy); only the first ray's origin is copied ahead for the "
                        "start-cell query") if args.transfer == "zero_copy" else
                       "InferScene.render_host: pinned host rays in, f16 rgba out, row bands "
                       "pipelined over two copy streams"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic,
                     "peak_source": peak_src,
                     "bytes_per_ray": b_ray,
                     "algorithmic_bytes_per_launch": alg,
                     "formula": "B_ray = 40 + 28*steps + 8*faces + 64*textured (traversal "
                                "means per ray); achieved = B_ray * rays / kernel_ms",
                     "kernel": "vt::infer_kernel<8, TexF16x4<8>>",
                     "kernel_ms": trace_ms},
        "compulsory_roofline": {"achieved": comp_achieved, "peak": hbm, "unit": "GB/s",
                                "frac": comp_achieved / hbm, "bytes_per_launch": comp,
                                "what": "every visited cell's data once (16-B face rows, site, "
                                        "density, texels) plus per-ray I/O"},
        "issue_roofline": issue,
        "traversal": stats,
        "clocks": clocks,
        # value loop: BVH query + trace; e2e loop: one BVH query + one trace per band
        "gpu_launches": 2 * args.steps + (1 + n_bands) * args.steps,
    }
    if not args.no_train_leg:
        out["training"] = training_leg(ws, rank, dev, min(args.steps, 10), args.allreduce)
    if not args.no_cpu_baseline and ws == 1:
        import oracle

        st = int(oracle.nn_query(s["points"], rays_np.reshape(-1, 6)[:1, :3])[0])
        thr = oracle.max_threads()
        rate, n, dt, _ = cpu_oracle_rate(s, rays_np, st, budget_s=15.0, threads=thr)
        out["cpu_baseline"] = {"value": rate / 1e6, "unit": "Mrays/s", "cores": thr,
                               "kind": "port",
                               "sample": f"{n} of {nr} rays of the view (strided), {dt:.1f} s"}
    print(json.dumps(out), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
