"""The drop-in operator module on the calls the reference's model code makes.

tests/golden/make_dropin.py ran the reference's own ``VoroTracing`` and
``VoroTracingInfer`` (vorotracing/vorotracing.py) with an oracle-backed
``vorotracing.cuda`` and recorded every operator call: the arguments exactly
as the model code built them (activated density, uint32 CSR with tail
padding, broadcast start cells, depth quantiles, the 4x8 tile permutation,
the Morton-sorted fp16 / q8 attributes, the q8 scale and offset as Python
floats), the upstream gradients autograd handed to the backward, the error
box's ray_error / cell_distortion_gate, and the results.  Here each call is
replayed through ``vorotracing_b200.cuda`` on the GPU:

* prefetch_octmap_adj returns the reference's (E+32, 4) float16 array, equal
  to the recorded one row for row over the CSR;
* trace_octmap_infer / trace_octmap_infer_q8 given that array (and, as well,
  a plain copy of the recorded array) return the recorded pixels bit for bit;
* TraceVoroTracing.apply returns the recorded rgba, depth and distortion bit
  for bit and, on backward with the recorded upstream gradients, the recorded
  gradients (relative 1e-3, the gradients are atomic sums), including the
  two-pass cell_distortion_gate step and the error box's point_error;
* NNBVH.query returns the recorded start cells.

The large texture arrays are regenerated from the recorder's seed and
checked against its SHA-256 digests before use.
"""
import os
import sys

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_dropin as MD  # noqa: E402

Z = np.load(os.path.join(HERE, "golden", "dropin_calls.npz"))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _get(k, name):
    return Z[f"{k}.{name}"]


def _has(k, name):
    return f"{k}.{name}" in Z.files


@pytest.fixture(scope="module")
def inputs():
    pts, dif, spe, den = MD.scene_inputs()
    assert list(Z["scene.sha"]) == [MD.sha(pts), MD.sha(dif), MD.sha(spe), MD.sha(den)]
    return pts, dif, spe, den


def _textures(kind, dif, spe):
    """The Morton-sorted attributes VoroTracingInfer built, from the seed."""
    perm = Z[f"morton_perm_{kind}"]
    if kind == "fp16":
        d = oracle.pad_f16x4(dif, MD.RES)[perm]
        s = oracle.pad_f16x4(spe, MD.RES)[perm]
        return d, s, None
    dq, ds, do = oracle.quantize_u8(dif)
    sq, ss, so = oracle.quantize_u8(spe)
    return dq[perm], sq[perm], (ds, do, ss, so)


def test_bvh_query_start_cells():
    from vorotracing_b200.cuda import NNBVH

    pts_by_sha = {}
    for k in ("train0", "train1", "infer_f16_0", "infer_q8_0"):
        p = _get(k, "points")
        pts_by_sha[MD.sha(p)] = p
    i = 0
    while _has(f"bvh_query{i}", "out"):
        k = f"bvh_query{i}"
        pts = pts_by_sha[str(_get(k, "points_sha"))]
        bvh = NNBVH()
        bvh.build(_dev(pts))
        got = bvh.query(_dev(pts), _dev(_get(k, "queries")))
        np.testing.assert_array_equal(got.cpu().numpy().astype(np.int64),
                                      _get(k, "out").astype(np.int64))
        i += 1
    assert i == 4


@pytest.mark.parametrize("i", [0, 1])
def test_prefetch_octmap_adj_reference_layout(i):
    from vorotracing_b200 import cuda as ops

    k = f"prefetch{i}"
    offs = _get(k, "offsets")
    got = ops.prefetch_octmap_adj(_dev(_get(k, "points")), _dev(_get(k, "adjacency")), _dev(offs))
    ref = _get(k, "out")
    assert tuple(got.shape) == ref.shape and got.dtype == torch.float16
    e = int(offs[-1])
    g = got.cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(g[:e], ref[:e])
    assert not g[e:].any()  # rows the reference leaves uninitialised are zero here


@pytest.mark.parametrize("kind", ["fp16", "q8"])
@pytest.mark.parametrize("adj_src", ["prefetched", "recorded_copy"])
def test_infer_replay(inputs, kind, adj_src):
    from vorotracing_b200 import cuda as ops

    pts, dif, spe, den = inputs
    k = "infer_f16_0" if kind == "fp16" else "infer_q8_0"
    d, s, q8 = _textures(kind, dif, spe)
    assert MD.sha(d) == str(_get(k, "diffuse_sha")) and MD.sha(s) == str(_get(k, "specular_sha"))
    if q8 is not None:
        np.testing.assert_array_equal(np.array(q8, np.float64), _get(k, "q8"))
    a = {n: _dev(_get(k, n)) for n in ("points", "density", "adjacency", "offsets", "rays",
                                       "start_point")}
    if adj_src == "prefetched":
        adj_diff = ops.prefetch_octmap_adj(a["points"], a["adjacency"], a["offsets"])
    else:
        adj_diff = _dev(_get(k, "adjacent_diff")).view(torch.float16)
    wt, mi, skip = _get(k, "scalars")
    if kind == "fp16":
        rgba = ops.trace_octmap_infer(a["points"], _dev(d), _dev(s), a["density"], a["adjacency"],
                                      a["offsets"], a["rays"], a["start_point"], adj_diff,
                                      _dev(_get(k, "ray_perm")), float(wt), int(mi), float(skip))
    else:
        qs = [float(v) for v in _get(k, "q8")]  # Python floats, as the model code passes them
        rgba = ops.trace_octmap_infer_q8(a["points"], _dev(d), _dev(s), a["density"],
                                         a["adjacency"], a["offsets"], a["rays"],
                                         a["start_point"], adj_diff, *qs, float(wt), int(mi),
                                         float(skip))
    torch.cuda.synchronize()
    assert tuple(rgba.shape) == tuple(_get(k, "rays").shape[:-1]) + (4,)
    got = rgba.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1, 4)
    np.testing.assert_array_equal(got, _get(k, "out_rgba"))


def _close(got, ref, name, rtol=1e-3, abs_frac=1e-4):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    scale = max(float(np.abs(ref).max()), 1e-30)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=abs_frac * scale, err_msg=name)


@pytest.mark.parametrize("step", [0, 1], ids=["plain", "distortion_gate"])
def test_trace_vorotracing_replay(inputs, step):
    from vorotracing_b200 import cuda as ops

    pts, dif, spe, den = inputs
    k = f"train{step}"
    assert str(_get(k, "diffuse_dtype")) == "torch.float32"
    assert MD.sha(dif) == str(_get(k, "diffuse_sha")) and MD.sha(spe) == str(_get(k, "specular_sha"))
    params = [_dev(_get(k, "points")).requires_grad_(), _dev(dif).requires_grad_(),
              _dev(spe).requires_grad_(), _dev(_get(k, "density")).requires_grad_()]
    wt, mi, rc = _get(k, "scalars")
    rgba, depth, contrib, n_int, errbox, dist = ops.TraceVoroTracing.apply(
        *params, _dev(_get(k, "adjacency")), _dev(_get(k, "offsets")), _dev(_get(k, "rays")),
        _dev(_get(k, "start_point")), _dev(_get(k, "depth_quantiles")), float(wt), int(mi),
        bool(rc))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(rgba.detach().cpu().numpy().reshape(-1, 4), _get(k, "out_rgba"))
    np.testing.assert_array_equal(depth.detach().cpu().numpy().reshape(-1, 2), _get(k, "out_depth"))
    np.testing.assert_array_equal(dist.detach().cpu().numpy().reshape(-1),
                                  _get(k, "out_distortion"))
    np.testing.assert_array_equal(n_int.detach().cpu().numpy().reshape(-1).astype(np.int64),
                                  _get(k, "out_n").astype(np.int64))
    np.testing.assert_allclose(contrib.detach().float().cpu().numpy().reshape(-1),
                               _get(k, "out_contribution"), rtol=1e-5, atol=1e-6)
    errbox.ray_error = _dev(_get(k, "ray_error"))
    if _has(k, "cell_distortion_gate"):
        errbox.cell_distortion_gate = _dev(_get(k, "cell_distortion_gate"))
    torch.autograd.backward(
        [rgba, depth, contrib, dist],
        [_dev(_get(k, "grad_rgba")), _dev(_get(k, "grad_depth")),
         _dev(_get(k, "grad_contribution")), _dev(_get(k, "grad_distortion"))])
    torch.cuda.synchronize()
    for p, name in zip(params, ("points", "diffuse", "specular", "density")):
        _close(p.grad.cpu().numpy(), _get(k, "grad_out_" + name), name)
    _close(errbox.point_error.float().cpu().numpy(), _get(k, "point_error"), "point_error")


def test_v3_foam_with_prefetched_adj_diff(inputs, tmp_path):
    """A V3 .foam written with the array prefetch_octmap_adj returns (as the
    reference's exporter writes model.adjacent_diff) carries the reference's
    adjacent_diff blob and renders the recorded pixels after reading back."""
    from vorotracing_b200 import cuda as ops
    from vorotracing_b200.formats import read_foam, write_foam

    pts, dif, spe, den = inputs
    k = "infer_f16_0"
    d, s, _ = _textures("fp16", dif, spe)
    p, adj, offs = _get(k, "points"), _get(k, "adjacency"), _get(k, "offsets")
    adj_diff = ops.prefetch_octmap_adj(_dev(p), _dev(adj), _dev(offs))
    pose = np.eye(4, dtype=np.float32)[:3][None]
    path = tmp_path / "scene_v3.foam"
    write_foam(path, p, _get(k, "density"), d, s, adj, offs, pose, MD.RES, MD.RES,
               adjacent_diff=adj_diff.cpu().numpy(), version=3)
    f = read_foam(path)
    e = int(offs[-1])
    assert f["adjacent_diff"].shape == _get("prefetch0", "out").shape
    np.testing.assert_array_equal(f["adjacent_diff"].view(np.uint16)[:e],
                                  _get("prefetch0", "out")[:e])
    wt, mi, skip = _get(k, "scalars")
    rgba = ops.trace_octmap_infer(
        _dev(f["points"]), _dev(f["diffuse_h4"]), _dev(f["specular_h4"]), _dev(f["density"]),
        _dev(f["adj"]), _dev(f["offs"]), _dev(_get(k, "rays")), _dev(_get(k, "start_point")),
        _dev(f["adjacent_diff"]), _dev(_get(k, "ray_perm")), float(wt), int(mi), float(skip))
    torch.cuda.synchronize()
    got = rgba.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1, 4)
    np.testing.assert_array_equal(got, _get(k, "out_rgba"))
