"""On-disk scene formats of VoroTracing, read and written without the reference.

* Checkpoint (``torch.save`` dict, vorotracing/vorotracing.py:421-436): keys
  ``xyz`` (N,3) f32, ``density`` (N,1) f32 *pre-activation* parameter (the
  model renders ``activation_scale * exp(density)``), ``adjacency`` and
  ``adjacency_offsets`` int64 CSR, ``color_diffuse`` / ``color_specular``
  (N, 3R^2) f32 logits.  ``VoroTracing.from_pretrained`` loads what
  ``save_checkpoint`` writes.
* ``.foam`` flat binary scene for external viewers, versions 4 and 3
  (scripts/export_for_viewer.py:17-51 and its writer :146-216): a 120-byte
  little-endian header, then points, density (activated), diffuse and
  specular octmaps in binary16 (3 channels per texel in V4, 4 in V3), CSR
  adjacency and offsets, V3's half4 adjacent_diff rows, and camera poses.
  ``read_foam`` returns arrays ready for ``render.InferScene`` /
  ``cuda.trace_octmap_infer`` (octmaps re-padded to Half4Texel rows); the
  packed face rows are rebuilt on the GPU by ``prefetch_octmap_adj``.
"""
from __future__ import annotations

import struct

import numpy as np

FOAM_MAGIC = 0x464F414D
_HEADER = struct.Struct("<IIIIIIIIffI")  # 44 bytes, then pose(48) aabb(24) has_specular(4)
HEADER_BYTES = 120


# ---------------------------------------------------------------- checkpoint

def save_checkpoint(path, points, density_param, adjacency, offsets, diffuse, specular):
    """Write the reference's checkpoint dict.  ``density_param`` is the
    pre-activation density (log of the rendered density at scale 1)."""
    import torch

    t = lambda a, dt: torch.as_tensor(np.asarray(a), dtype=dt).cpu()
    n = int(np.asarray(points).shape[0])
    torch.save({
        "xyz": t(points, torch.float32).reshape(n, 3),
        "density": t(density_param, torch.float32).reshape(n, 1),
        "adjacency": t(np.asarray(adjacency).astype(np.int64), torch.int64),
        "adjacency_offsets": t(np.asarray(offsets).astype(np.int64), torch.int64),
        "color_diffuse": t(diffuse, torch.float32).reshape(n, -1),
        "color_specular": t(specular, torch.float32).reshape(n, -1),
    }, path)


def load_checkpoint(path, activation_scale: float = 1.0) -> dict:
    """Arrays of a reference checkpoint; ``density`` is activated
    (``activation_scale * exp(param)``, vorotracing.py:346-347)."""
    import torch

    d = torch.load(path, map_location="cpu")
    dens = activation_scale * torch.exp(d["density"].float())
    return {
        "points": d["xyz"].float().numpy(),
        "density": dens.numpy(),
        "adj": d["adjacency"].numpy().astype(np.uint32),
        "offs": d["adjacency_offsets"].numpy().astype(np.uint32),
        "diffuse": d["color_diffuse"].float().numpy(),
        "specular": d["color_specular"].float().numpy(),
    }


# ---------------------------------------------------------------- .foam

def _rgb_to_half4(rgb16: np.ndarray, n: int, res: int) -> np.ndarray:
    out = np.zeros((n, res * res, 4), np.float16)
    out[:, :, :3] = rgb16.reshape(n, res * res, 3)
    return out.reshape(n, res * res * 4)


def write_foam(path, points, density, diffuse_h4, specular_h4, adjacency, offsets, poses,
               res_diff: int, res_spec: int, weight_threshold=0.001, cell_skip_threshold=0.0,
               max_intersections=1024, aabb=None, adjacent_diff=None, version: int = 4):
    """Write a .foam scene.  ``density`` is the activated density; octmaps are
    (N, 4R^2) binary16 Half4Texel rows (pass ``specular_h4=None`` for a
    diffuse-only file); ``poses`` (P, 3, 4) camera-to-world, poses[0] is the
    default view; ``adjacent_diff`` (E', 4) binary16 is required for V3."""
    pts = np.ascontiguousarray(points, np.float32)
    n = pts.shape[0]
    dens = np.ascontiguousarray(density, np.float32).reshape(-1)
    adj = np.ascontiguousarray(adjacency, np.uint32)
    offs = np.ascontiguousarray(offsets, np.uint32)
    poses = np.ascontiguousarray(poses, np.float32).reshape(-1, 3, 4)
    dif = np.ascontiguousarray(diffuse_h4, np.float16).reshape(n, res_diff * res_diff * 4)
    has_spec = specular_h4 is not None
    spe = None
    if has_spec:
        spe = np.ascontiguousarray(specular_h4, np.float16).reshape(n, res_spec * res_spec * 4)
    else:
        res_spec = 0
    if version >= 4:
        dif = dif.reshape(n, -1, 4)[:, :, :3].reshape(n, -1)
        if has_spec:
            spe = spe.reshape(n, -1, 4)[:, :, :3].reshape(n, -1)
        adj_diff_size = 0
    else:
        adjacent_diff = np.ascontiguousarray(adjacent_diff, np.float16)
        adj_diff_size = adjacent_diff.shape[0]
    if aabb is None:
        aabb = (pts.min(0), pts.max(0))
    with open(path, "wb") as f:
        f.write(_HEADER.pack(FOAM_MAGIC, version, n, poses.shape[0], adj.shape[0], adj_diff_size,
                             res_diff, res_spec, float(weight_threshold),
                             float(cell_skip_threshold), int(max_intersections)))
        f.write(poses[0].tobytes())
        f.write(np.asarray(aabb[0], np.float32).tobytes())
        f.write(np.asarray(aabb[1], np.float32).tobytes())
        f.write(struct.pack("<I", 1 if has_spec else 0))
        for blob in (pts, dens, dif, spe, adj, offs):
            if blob is not None:
                f.write(blob.tobytes())
        if version < 4:
            f.write(adjacent_diff.tobytes())
        f.write(poses.tobytes())


def read_foam(path) -> dict:
    """Parse a V3 or V4 .foam file.  Octmaps come back as Half4Texel rows."""
    buf = memoryview(open(path, "rb").read())
    (magic, version, n, n_poses, adj_size, adj_diff_size, rd, rs, wt, skip,
     max_int) = _HEADER.unpack_from(buf, 0)
    if magic != FOAM_MAGIC:
        raise ValueError(f"not a .foam file (magic {magic:#x})")
    if version not in (3, 4):
        raise ValueError(f"unsupported .foam version {version}")
    o = _HEADER.size
    take = lambda dt, count: np.frombuffer(buf, dt, count, o)
    default_pose = take(np.float32, 12).reshape(3, 4).copy(); o += 48
    aabb_min = take(np.float32, 3).copy(); o += 12
    aabb_max = take(np.float32, 3).copy(); o += 12
    (has_spec,) = struct.unpack_from("<I", buf, o); o += 4
    assert o == HEADER_BYTES
    ch = 3 if version >= 4 else 4

    def blob(dt, count):
        nonlocal o
        a = np.frombuffer(buf, dt, count, o).copy()
        o += a.nbytes
        return a

    pts = blob(np.float32, n * 3).reshape(n, 3)
    dens = blob(np.float32, n).reshape(n, 1)
    dif = blob(np.float16, n * rd * rd * ch).reshape(n, -1)
    spe = blob(np.float16, n * rs * rs * ch).reshape(n, -1) if has_spec else None
    adj = blob(np.uint32, adj_size)
    offs = blob(np.uint32, n + 1)
    adj_diff = blob(np.float16, adj_diff_size * 4).reshape(-1, 4) if version < 4 else None
    poses = blob(np.float32, n_poses * 12).reshape(n_poses, 3, 4)
    if o != len(buf):
        raise ValueError(f".foam size mismatch: parsed {o} of {len(buf)} bytes")
    if ch == 3:
        dif = _rgb_to_half4(dif, n, rd)
        if spe is not None:
            spe = _rgb_to_half4(spe, n, rs)
    if spe is None:  # diffuse-only file: a zero specular map keeps the kernels' layout
        spe = np.zeros_like(dif)
        rs = rd
    return dict(version=version, points=pts, density=dens, diffuse_h4=dif, specular_h4=spe,
                res_diff=rd, res_spec=rs, has_specular=bool(has_spec), adj=adj, offs=offs,
                adjacent_diff=adj_diff, poses=poses, default_pose=default_pose,
                aabb=(aabb_min, aabb_max), weight_threshold=wt, cell_skip_threshold=skip,
                max_intersections=max_int)
