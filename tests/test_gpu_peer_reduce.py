"""The training step's gradient all-reduce over peer memory
(vt_grad_allreduce_peer), with the ranks emulated on one GPU.

Each emulated rank runs the backward of its own rays with
VT_BWD_KEEP_WORKSPACE into its own workspace and bucket; then every rank's
call of the kernel (in turn, on one stream: the kernel never waits on
another rank) must leave every bucket equal, bit for bit, to the rank-order
sum of the ranks' compacted gradients (read from their workspaces, as the
ordinary backward's compaction pass would write them).  The kernel sees device addresses only, so local
buffers stand in for the peers' IPC-mapped ones; the cross-process mapping
is exercised by ``bench.py --gpus N``.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("world", [1, 2, 3])
def test_peer_allreduce_matches_rank_order_sum(c1_scene, c1_rays, world):
    from vorotracing_b200 import _lib
    from vorotracing_b200.cuda import _ops
    from vorotracing_b200.shard import GradBucket

    s = c1_scene
    res = s["res"]
    rays = c1_rays.reshape(-1, 6)
    st = int(oracle.nn_query(s["points"], rays[:1, :3])[0])
    scene = (_dev(s["points"]), _dev(s["diffuse"]), _dev(s["specular"]), _dev(s["density"]),
             _dev(s["adj"]), _dev(s["offs"]))
    n = s["points"].shape[0]
    L = _lib.lib()
    wsb = int(L.vt_trace_bwd_workspace_bytes(C.c_uint32(n), C.c_int(res)))
    ntex = n * res * res
    a256 = lambda x: (x + 255) // 256 * 256
    buckets, wss, expect = [], [], []
    for r in range(world):
        rr = _dev(rays[r::world])
        start = torch.full((rr.size(0),), st, dtype=torch.int32, device="cuda").view(torch.uint32)
        args = (*scene, rr, start)
        f = _ops.trace_vorotracing_fwd(*args, None, 0.01, 1024, False)
        g = torch.randn(f[0].shape, generator=torch.Generator("cuda").manual_seed(10 + r),
                        device="cuda")
        common = (f[0], g, None, None, None, None, 0.0, f[5], None, f[6], f[7], f[8], 0.01, 1024)
        b = GradBucket(n, s["diffuse"].shape[1], "cuda")
        b.flat.fill_(7.0)  # every word is overwritten by the reduction
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        _ops.trace_vorotracing_bwd(*args, *common, grads=b.views(), accumulate=False,
                                   workspace=ws, keep_workspace=True)
        # this rank's compacted gradients, read from the workspace it kept:
        # padded float4 rows (x, y, z, unused) for diffuse, specular, sites
        wf = ws.view(torch.float32)
        take = lambda off, rows: wf[off // 4: off // 4 + rows * 4].view(rows, 4)[:, :3].reshape(-1)
        e = torch.cat([take(2 * a256(ntex * 16), n), b.density.reshape(-1).clone(),
                       take(0, ntex), take(a256(ntex * 16), ntex)])
        buckets.append(b)
        wss.append(ws)
        expect.append(e)
    want = expect[0].clone()
    for r in range(1, world):
        want += expect[r]
    slot = int(L.vt_peer_staging_floats(C.c_uint32(n), C.c_int(res), C.c_uint32(world)))
    stagings = [torch.full((world * slot,), float("nan"), device="cuda") for _ in range(world)]
    g = _lib.VtPeerGrads()
    g.world, g.num_points, g.res = world, n, res
    for k in range(world):
        g.workspace[k] = wss[k].data_ptr()
        g.bucket[k] = buckets[k].flat.data_ptr()
        g.staging[k] = stagings[k].data_ptr()
    for phase in (0, 1):  # every rank's phase 0 before any phase 1
        for r in range(world):
            _lib.check(L.vt_grad_allreduce_peer(C.byref(g), C.c_uint32(r), C.c_uint32(phase),
                                                _lib.stream_ptr()), "vt_grad_allreduce_peer")
    torch.cuda.synchronize()
    assert want.abs().sum() > 0
    for b in buckets:
        assert torch.equal(b.flat.view(torch.int32), want.view(torch.int32))


def test_peer_allreduce_rejects_bad_arguments():
    from vorotracing_b200 import _lib

    L = _lib.lib()
    g = _lib.VtPeerGrads()
    g.world, g.num_points, g.res = 9, 10, 8
    assert L.vt_grad_allreduce_peer(C.byref(g), C.c_uint32(0), C.c_uint32(0), None) != 0
    assert b"world" in L.vt_last_error()
    g.world = 2
    assert L.vt_grad_allreduce_peer(C.byref(g), C.c_uint32(2), C.c_uint32(0), None) != 0
    assert b"rank" in L.vt_last_error()
    assert L.vt_grad_allreduce_peer(C.byref(g), C.c_uint32(0), C.c_uint32(2), None) != 0
    assert b"phase" in L.vt_last_error()
    assert L.vt_grad_allreduce_peer(C.byref(g), C.c_uint32(0), C.c_uint32(0), None) != 0
    assert b"buffers missing" in L.vt_last_error()
