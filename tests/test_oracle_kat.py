"""Known-answer tests that pin the CPU oracle to closed-form results.

The reference ships no tests or fixtures, so the oracle is pinned by scenes
whose traversal is analytic: sites on an integer lattice have unit-cube
Voronoi cells with faces at half-integers, so a ray's exit distances,
segment lengths, transmittance, colour and depth quantiles follow in closed
form (reference semantics: tracing_octmap.cu:39-123,
ray_integrator_octmap.cuh:102-152 and :315-344).
"""
import numpy as np
import pytest

import oracle

G = 5  # lattice is G x G x G


def lattice_scene(sigma=0.7, logit=0.3, res=4):
    idx = lambda i, j, k: (i * G + j) * G + k
    pts, adj, offs = [], [], [0]
    for i in range(G):
        for j in range(G):
            for k in range(G):
                pts.append((i, j, k))
                for d in ((1, 0, 0), (-1, 0, 0), (0, 1, 0), (0, -1, 0), (0, 0, 1), (0, 0, -1)):
                    a, b, c = i + d[0], j + d[1], k + d[2]
                    if 0 <= a < G and 0 <= b < G and 0 <= c < G:
                        adj.append(idx(a, b, c))
                offs.append(len(adj))
    n = len(pts)
    adj = np.array(adj + [0] * 32, np.uint32)
    dif = np.full((n, 3 * res * res), logit, np.float32)
    spe = np.full((n, 3 * res * res), -0.1, np.float32)
    den = np.full((n, 1), sigma, np.float32)
    return np.array(pts, np.float32), adj, np.array(offs, np.uint32), den, dif, spe, idx


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


@pytest.mark.parametrize("attr", [oracle.ATTR_F32, oracle.ATTR_F16])
def test_axis_ray_closed_form(attr):
    sigma, logit = 0.7, 0.3
    pts, adj, offs, den, dif, spe, idx = lattice_scene(sigma, logit)
    if attr == oracle.ATTR_F16:
        dif, spe = dif.astype(np.float16), spe.astype(np.float16)
    S = oracle.Scene(pts, adj, offs, den, dif, spe, attr)
    o = np.array([0.1, 0.2, 0.3], np.float32)
    ray = np.array([[*o, 2.0, 0.0, 0.0]], np.float32)  # direction is normalised by the kernel
    r = oracle.trace_fwd(S, ray, [idx(0, 0, 0)], depth_quantiles=np.float32([[0.5, 0.2]]),
                         wt=0.0, seq_cap=16)
    # cells (0..4,0,0); exits at x = 0.5, 1.5, 2.5, 3.5; the last cell has no exit
    assert list(r["seq"][0, : r["seq_len"][0]]) == [idx(i, 0, 0) for i in range(5)]
    assert r["n"][0] == 5
    L = 3.5 - 0.1
    T = np.exp(-sigma * L)
    c = _sig(logit - 0.1)
    rgba = np.asarray(r["rgba"], np.float64)[0]
    tol = 1e-6 if attr == oracle.ATTR_F32 else 2e-3
    np.testing.assert_allclose(rgba[:3], c * (1 - T), atol=tol)
    np.testing.assert_allclose(rgba[3], 1 - T, atol=tol)
    # depth quantiles: T(t) = exp(-sigma t) crosses q at t = log(1/q)/sigma
    np.testing.assert_allclose(r["depth"][0], np.log(1 / np.float64([0.5, 0.2])) / sigma, rtol=1e-5)
    assert list(r["depth_idx"][0]) == [idx(int(np.floor(0.1 + np.log(2) / sigma + 0.5)), 0, 0),
                                       idx(int(np.floor(0.1 + np.log(5) / sigma + 0.5)), 0, 0)]
    np.testing.assert_allclose(r["t_far"][0], 3.4, rtol=1e-6)
    np.testing.assert_allclose(r["W"][0], 1 - T, rtol=1e-5)


def test_weight_threshold_stops_in_closed_form_cell():
    sigma = 2.0
    pts, adj, offs, den, dif, spe, idx = lattice_scene(sigma)
    S = oracle.Scene(pts, adj, offs, den, dif, spe, oracle.ATTR_F32)
    ray = np.array([[0.0, 0.0, 0.0, 1.0, 0.0, 0.0]], np.float32)
    wt = 0.01
    r = oracle.trace_fwd(S, ray, [idx(0, 0, 0)], wt=wt, seq_cap=16)
    # T after cell i (exit at x = i + 0.5) is exp(-sigma (i + 0.5)); stop when T <= wt
    i_stop = int(np.ceil(np.log(1 / wt) / sigma - 0.5))
    assert r["seq_len"][0] == i_stop + 1
    np.testing.assert_allclose(r["rgba"][0, 3], 1 - np.exp(-sigma * (i_stop + 0.5)), rtol=1e-6)


def test_infer_density_gate_and_skip():
    """infer leaves T untouched in cells with density <= 1e-6
    (ray_integrator_octmap.cuh:323-327) and skips colour below the skip weight."""
    pts, adj, offs, den, dif, spe, idx = lattice_scene(0.5)
    den = den.copy()
    den[idx(1, 0, 0)] = 0.0
    pad = lambda a: np.concatenate([a.reshape(len(a), -1, 3),
                                    np.zeros((len(a), a.shape[1] // 3, 1), np.float32)], -1)
    d4 = pad(dif).astype(np.float16).reshape(len(dif), -1)
    s4 = pad(spe).astype(np.float16).reshape(len(spe), -1)
    S = oracle.Scene(pts, adj, offs, den, d4, s4, oracle.ATTR_F16X4)
    ray = np.array([[0.0, 0.0, 0.0, 1.0, 0.0, 0.0]], np.float32)
    r = oracle.trace_infer(S, ray, [idx(0, 0, 0)], wt=0.0, skip=0.0)
    L = 0.5 + 1.0 + 1.0  # cells 0, 2, 3 integrate; cell 1 is empty; cell 4 has no exit
    np.testing.assert_allclose(float(r["rgba"][0, 3]), 1 - np.exp(-0.5 * L), atol=1e-3)
    assert r["stats"][0, 3] == 3
    r2 = oracle.trace_infer(S, ray, [idx(0, 0, 0)], wt=0.0, skip=0.5)
    assert r2["stats"][0, 3] == 0 and float(r2["rgba"][0, 0]) == 0.0


def test_max_intersections_counts_steps():
    pts, adj, offs, den, dif, spe, idx = lattice_scene(0.1)
    S = oracle.Scene(pts, adj, offs, den, dif, spe, oracle.ATTR_F32)
    ray = np.array([[0.0, 0.0, 0.0, 1.0, 0.0, 0.0]], np.float32)
    for m, n_expect, cells in [(1, 2, 1), (2, 3, 2), (10, 5, 5)]:
        r = oracle.trace_fwd(S, ray, [idx(0, 0, 0)], wt=0.0, max_int=m, seq_cap=16)
        assert r["n"][0] == n_expect and r["seq_len"][0] == cells


def test_nn_query_ties_to_lowest_index():
    pts = np.float32([[1, 0, 0], [-1, 0, 0], [0, 0, 0], [0, 0, 0]])
    q = np.float32([[0, 0, 0], [0.5, 0, 0], [10, 0, 0]])
    np.testing.assert_array_equal(oracle.nn_query(pts, q), [2, 0, 0])
