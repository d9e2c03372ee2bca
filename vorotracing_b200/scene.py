"""Seeded synthetic Voronoi scenes and cameras for the benchmark configurations.

The reference measures on Mip-NeRF 360 captures, which are not available here;
these generators stand in for them with the shapes, sizes and value
distributions of the benchmark configurations:

* C1: 16,384 sites, 70 % on a noisy unit sphere (sigma 0.01), 30 % uniform in
  [-2, 2]^3; density softplus(N(0,1)); 4x4 octahedral diffuse U(0,1).
* C2/C3: 1M sites, 70 % surface split between the noisy sphere and the ground
  plane z = -1 over [-2, 2]^2, 30 % uniform; 8x8 textures.
* C4/C5: the same mixture at 3M / 4M sites.

Adjacency is the Delaunay graph (= Voronoi face adjacency) from
scipy.spatial.Delaunay, stored as the reference's uint32 CSR with 32 padding
entries at the tail (vorotracing/cuda/__init__.py:39-45).

Cameras follow the reference's ``generate_camera_rays``
(vorotracing/utils/__init__.py:85-130): OpenCV axes (x right, y down, z
forward), integer pixel coordinates, K = [[f, 0, W/2], [0, f, H/2], [0, 0, 1]].
"""
from __future__ import annotations

import hashlib
import os

import numpy as np

CSR_PAD = 32


def softplus(x):
    return np.logaddexp(0.0, x)


def make_sites(n: int, seed: int, plane: bool) -> np.ndarray:
    """Surface/uniform mixture of ``n`` sites (float32, (n, 3))."""
    rng = np.random.default_rng(seed)
    n_surf = int(round(0.7 * n))
    n_uni = n - n_surf
    if plane:
        n_sph = n_surf // 2
        n_pl = n_surf - n_sph
    else:
        n_sph, n_pl = n_surf, 0
    d = rng.standard_normal((n_sph, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    sph = d + rng.normal(0.0, 0.01, (n_sph, 3))
    pl = np.stack([rng.uniform(-2, 2, n_pl), rng.uniform(-2, 2, n_pl),
                   -1.0 + rng.normal(0.0, 0.01, n_pl)], axis=1)
    uni = rng.uniform(-2, 2, (n_uni, 3))
    pts = np.concatenate([sph, pl, uni], 0)
    pts = pts[rng.permutation(n)]
    return pts.astype(np.float32)


def delaunay_csr(points: np.ndarray, pad: int = CSR_PAD):
    """Delaunay neighbours as (adjacency uint32 (E+pad,), offsets uint32 (N+1,))."""
    from scipy.spatial import Delaunay

    tri = Delaunay(points.astype(np.float64))
    indptr, ind = tri.vertex_neighbor_vertices
    adj = np.zeros(len(ind) + pad, np.uint32)
    adj[: len(ind)] = ind
    return adj, indptr.astype(np.uint32)


def _cache_path(tag: str) -> str:
    root = os.environ.get("VT_SCENE_CACHE", os.path.join(os.path.expanduser("~"), ".cache",
                                                        "vorotracing_b200"))
    os.makedirs(root, exist_ok=True)
    return os.path.join(root, tag + ".npz")


def gpu_voronoi_csr(points: np.ndarray, pad: int = CSR_PAD):
    """Voronoi adjacency built on the GPU (cuda.build_voronoi_adjacency)."""
    import torch

    from .cuda import build_voronoi_adjacency

    adj, offs, _ = build_voronoi_adjacency(torch.from_numpy(np.ascontiguousarray(points)).cuda(),
                                           chunk_padding=pad)
    return adj.cpu().numpy(), offs.cpu().numpy()


def make_scene(n: int, seed: int, plane: bool, res: int, cache: bool = True,
               adjacency: str = "qhull") -> dict:
    """Sites, CSR and attributes.  Attributes are float32 logits:
    diffuse U(0,1), specular U(-0.5,0.5) (N, 3R^2); density softplus(N(0,1)) (N, 1).
    adjacency: "qhull" (scipy Delaunay, the parity tests' scenes) or "gpu"
    (the GPU clipping builder, seconds instead of minutes for millions of sites)."""
    tag = hashlib.sha1(f"v1-{n}-{seed}-{plane}-{adjacency}".encode()).hexdigest()[:16]
    path = _cache_path(tag)
    if cache and os.path.exists(path):
        z = np.load(path)
        pts, adj, offs = z["points"], z["adj"], z["offs"]
    else:
        pts = make_sites(n, seed, plane)
        adj, offs = delaunay_csr(pts) if adjacency == "qhull" else gpu_voronoi_csr(pts)
        if cache:
            np.savez(path, points=pts, adj=adj, offs=offs)
    rng = np.random.default_rng(seed + 1000)
    density = softplus(rng.standard_normal((n, 1))).astype(np.float32)
    diffuse = rng.uniform(0, 1, (n, 3 * res * res)).astype(np.float32)
    specular = rng.uniform(-0.5, 0.5, (n, 3 * res * res)).astype(np.float32)
    return dict(points=pts, adj=adj, offs=offs, density=density, diffuse=diffuse,
                specular=specular, res=res)


CONFIGS = {
    "C1": dict(n=16384, seed=0, plane=False, res=4, W=128, H=128),
    "C2": dict(n=1_000_000, seed=1, plane=True, res=8, W=1296, H=840),
    "C3": dict(n=1_000_000, seed=1, plane=True, res=8, W=1296, H=840),
    "C4": dict(n=3_000_000, seed=3, plane=True, res=8, W=1552, H=1040),
    "C5": dict(n=4_000_000, seed=4, plane=True, res=8, W=1920, H=1080),
}


def config_scene(name: str, n: int | None = None, cache: bool = True,
                 adjacency: str = "qhull") -> dict:
    c = CONFIGS[name]
    return make_scene(n or c["n"], c["seed"], c["plane"], c["res"], cache=cache,
                      adjacency=adjacency)


# ---------------------------------------------------------------- cameras

def look_at(eye, target=(0.0, 0.0, 0.0), up=(0.0, 0.0, 1.0)) -> np.ndarray:
    """Camera-to-world (4,4) with OpenCV axes: z forward, x right, y down."""
    eye = np.asarray(eye, np.float64)
    f = np.asarray(target, np.float64) - eye
    f /= np.linalg.norm(f)
    r = np.cross(f, np.asarray(up, np.float64))
    if np.linalg.norm(r) < 1e-9:
        r = np.cross(f, np.array([0.0, 1.0, 0.0]))
    r /= np.linalg.norm(r)
    d = np.cross(f, r)
    T = np.eye(4)
    T[:3, 0], T[:3, 1], T[:3, 2], T[:3, 3] = r, d, f, eye
    return T


def intrinsics(W: int, H: int, fov_y_deg: float = 60.0) -> np.ndarray:
    f = 0.5 * H / np.tan(0.5 * np.radians(fov_y_deg))
    return np.array([[f, 0, W / 2.0], [0, f, H / 2.0], [0, 0, 1.0]])


def orbit_pose(i: int, n: int, radius: float = 3.0, elev_deg: float = 15.0) -> np.ndarray:
    az = 2.0 * np.pi * i / n
    el = np.radians(elev_deg)
    eye = radius * np.array([np.cos(az) * np.cos(el), np.sin(az) * np.cos(el), np.sin(el)])
    return look_at(eye)


def pinhole_rays(K, T_c2w, W: int, H: int) -> np.ndarray:
    """(H, W, 6) float32 rays, the reference's generate_camera_rays convention
    evaluated in float32 (vorotracing/utils/__init__.py:85-130)."""
    K = np.asarray(K, np.float32)
    T = np.asarray(T_c2w, np.float32)
    u, v = np.meshgrid(np.arange(W, dtype=np.float32), np.arange(H, dtype=np.float32),
                       indexing="xy")
    x = (u - K[0, 2]) / K[0, 0]
    y = (v - K[1, 2]) / K[1, 1]
    dc = np.stack([x, y, np.ones_like(x)], -1)
    dc = dc / np.linalg.norm(dc, axis=-1, keepdims=True)
    dw = dc.reshape(-1, 3) @ T[:3, :3].T
    dw = dw / np.linalg.norm(dw, axis=-1, keepdims=True)
    o = np.broadcast_to(T[:3, 3], dw.shape)
    return np.concatenate([o, dw], -1).astype(np.float32).reshape(H, W, 6)


def config_rays(name: str, view: int = 0, n_views: int = 64) -> np.ndarray:
    c = CONFIGS[name]
    W, H = c["W"], c["H"]
    if name == "C1":
        T = look_at((0.0, 0.0, 3.0), up=(0.0, 1.0, 0.0))
    else:
        T = orbit_pose(view, n_views)
    return pinhole_rays(intrinsics(W, H), T, W, H)


def _main(argv=None):
    """python -m vorotracing_b200.scene voronoi <config> [--sites N] [--repeat K]

    Generates a configuration's sites and builds their Voronoi adjacency on
    the GPU, printing the build time and entry count (a profiling target)."""
    import argparse
    import time

    import torch

    from .cuda import build_voronoi_adjacency

    ap = argparse.ArgumentParser(prog="python -m vorotracing_b200.scene")
    ap.add_argument("what", choices=["voronoi"])
    ap.add_argument("config", choices=sorted(CONFIGS))
    ap.add_argument("--sites", type=int, default=None)
    ap.add_argument("--repeat", type=int, default=2)
    a = ap.parse_args(argv)
    c = CONFIGS[a.config]
    pts = torch.from_numpy(make_sites(a.sites or c["n"], c["seed"], c["plane"])).cuda()
    for _ in range(a.repeat):
        torch.cuda.synchronize()
        t = time.time()
        adj, offs, status = build_voronoi_adjacency(pts)
        torch.cuda.synchronize()
        print(f"{a.config}: {pts.size(0)} sites, {int(offs[-1])} entries, "
              f"{int(status[0])} unconverged, {time.time() - t:.3f} s", flush=True)


if __name__ == "__main__":
    _main()
