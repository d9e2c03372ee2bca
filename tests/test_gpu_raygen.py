"""Camera ray generation against float64 numpy restatements of each model."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lowbias32(x):
    x = np.uint64(x) & np.uint64(0xFFFFFFFF)
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & np.uint64(0xFFFFFFFF)
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & np.uint64(0xFFFFFFFF)
    x ^= x >> np.uint64(16)
    return x


def _rand(seed, pix, s, dim):
    h = _lowbias32(np.uint64(seed) ^ _lowbias32(np.uint64(pix) ^ _lowbias32(np.uint64(s * 4 + dim))))
    return float(h >> np.uint64(8)) / 16777216.0


def _ref(cam):
    R = np.asarray(cam.c2w, np.float64)[:3, :3]
    c = np.asarray(cam.c2w, np.float64)[:3, 3]
    out = np.zeros((cam.height, cam.width, cam.spp, 6))
    g = int(np.ceil(np.sqrt(cam.spp)))
    for v in range(cam.height):
        for u in range(cam.width):
            x, y = (u - cam.cx) / cam.fx, (v - cam.cy) / cam.fy
            for s in range(cam.spp):
                o = c.copy()
                if cam.model == 1:
                    r = np.hypot(x, y)
                    dc = np.array([np.sin(r) * x / r, np.sin(r) * y / r, np.cos(r)]) if r > 0 \
                        else np.array([0, 0, 1.0])
                elif cam.model == 2:
                    dc = np.array([x, y, 1.0])
                    o = c + np.asarray(cam.velocity) * (v / (cam.height - 1) * cam.rs_duration)
                elif cam.model == 3:
                    pix = v * cam.width + u
                    a = ((s % g) + _rand(cam.seed, pix, s, 0)) / g * 2 - 1
                    b = ((s // g) + _rand(cam.seed, pix, s, 1)) / g * 2 - 1
                    if abs(a) > abs(b):
                        rr, phi = a, np.pi / 4 * (b / a)
                    elif b != 0:
                        rr, phi = b, np.pi / 2 - np.pi / 4 * (a / b)
                    else:
                        rr, phi = 0.0, 0.0
                    lens = np.array([cam.lens_radius * rr * np.cos(phi),
                                     cam.lens_radius * rr * np.sin(phi), 0.0])
                    dc = np.array([x, y, 1.0]) * cam.focus_distance - lens
                    o = c + R @ lens
                else:
                    dc = np.array([x, y, 1.0])
                d = R @ (dc / np.linalg.norm(dc))
                out[v, u, s] = np.concatenate([o, d / np.linalg.norm(d)])
    return out


def _cams():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cameras import Camera

    T = sc.orbit_pose(3, 64)
    K = sc.intrinsics(24, 16)
    base = Camera.pinhole(K, T, 24, 16)
    fe = Camera.fisheye(T, 24, 16, 190.0)
    rs = Camera.pinhole(K, T, 24, 16)
    rs.model, rs.rs_duration, rs.velocity = 2, 0.03, (1.0, 0.0, 0.0)
    tl = Camera.pinhole(K, T, 24, 16)
    tl.model, tl.spp, tl.lens_radius, tl.focus_distance, tl.seed = 3, 4, 0.02, 3.0, 7
    return [base, fe, rs, tl]


@pytest.mark.parametrize("i", range(4))
def test_raygen_models(i):
    cam = _cams()[i]
    got = cam.rays().cpu().numpy().reshape(cam.height, cam.width, cam.spp, 6)
    np.testing.assert_allclose(got, _ref(cam), atol=3e-6, rtol=0)


def test_pinhole_matches_scene_helper():
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cameras import Camera

    T, K = sc.orbit_pose(5, 64), sc.intrinsics(64, 48)
    got = Camera.pinhole(K, T, 64, 48).rays().cpu().numpy()
    np.testing.assert_allclose(got, sc.pinhole_rays(K, T, 64, 48), atol=3e-7, rtol=0)


@pytest.mark.parametrize("model", [1, 3])
def test_per_ray_start_render_matches_oracle(c1_scene, model):
    """Non-pinhole rays with one BVH start cell per ray, against the oracle
    given the brute-force nearest site of every ray origin."""
    import oracle
    from vorotracing_b200 import scene as sc
    from vorotracing_b200.cameras import Camera
    from vorotracing_b200.render import InferScene

    s = c1_scene
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    scene = InferScene(d(s["points"]), d(s["density"]), d(s["adj"]), d(s["offs"]),
                       d(s["diffuse"]), d(s["specular"]))
    T = sc.look_at((0.0, 0.0, 3.0), up=(0.0, 1.0, 0.0))
    if model == 1:
        cam = Camera.fisheye(T, 48, 32, 190.0)
    else:
        cam = Camera.pinhole(sc.intrinsics(48, 32), T, 48, 32)
        cam.model, cam.spp, cam.lens_radius, cam.focus_distance, cam.seed = 3, 4, 0.3, 3.0, 9
    rays = cam.rays().reshape(-1, 6)
    rgba = scene.render(rays, weight_threshold=0.01, cell_skip_threshold=1e-3, per_ray_start=True)
    r = rays.cpu().numpy()
    start = oracle.nn_query(s["points"], r[:, :3]).astype(np.uint32)
    S = oracle.Scene(s["points"], s["adj"], s["offs"], s["density"],
                     oracle.pad_f16x4(s["diffuse"], 4), oracle.pad_f16x4(s["specular"], 4),
                     oracle.ATTR_F16X4)
    ref = oracle.trace_infer(S, r, start, wt=0.01, skip=1e-3)
    np.testing.assert_array_equal(rgba.cpu().numpy().view(np.uint16), ref["rgba"].view(np.uint16))
