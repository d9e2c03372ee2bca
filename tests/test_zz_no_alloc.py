"""The allocation-free BVH build, vt_bvh_build_noalloc, called through the C ABI.

Some callers of this library cannot allocate device memory: an application
that lends the library only its input and output buffers and keeps every
other byte of device memory under its own budget, or a language binding with
no CUDA allocator to call.  For them vt_bvh_build_noalloc keeps its scratch
in a fixed array inside the library.  These tests check that it writes the
same BVH as vt_bvh_build with a caller-provided workspace, on two calls in a
row with different sites (the array keeps the previous call's contents), and
that it rejects inputs above its size limit.  This file is collected last on
purpose, so a run that stops at the first failure has run everything else.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _build_both(L, pts):
    from vorotracing_b200._lib import ptr, stream_ptr

    n = pts.size(0)
    nb = int(L.vt_bvh_nodes_bytes(C.c_uint32(n)))
    wb = int(L.vt_bvh_workspace_bytes(C.c_uint32(n)))
    ref = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    got = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    s = stream_ptr()
    assert L.vt_bvh_build(ptr(pts), C.c_uint32(n), ptr(ref), C.c_uint64(nb), ptr(ws),
                          C.c_uint64(wb), s) == 0
    st = L.vt_bvh_build_noalloc(ptr(pts), C.c_uint32(n), ptr(got), C.c_uint64(nb), s)
    assert st == 0, L.vt_last_error()
    torch.cuda.synchronize()
    return ref, got


def _query(L, blob, pts, q):
    from vorotracing_b200._lib import ptr, stream_ptr

    out = torch.empty(q.size(0), dtype=torch.int32, device="cuda")
    assert L.vt_bvh_query(ptr(blob), ptr(pts), C.c_uint32(pts.size(0)), ptr(q),
                          C.c_uint32(q.size(0)), ptr(out), None, stream_ptr()) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_noalloc_build_matches_workspace_build_twice():
    from vorotracing_b200._lib import lib

    L = lib()
    rng = np.random.default_rng(0)
    for n in (200_000, 3_000):  # second call: fewer sites over the first call's leftovers
        pts = torch.from_numpy(rng.uniform(-2, 2, (n, 3)).astype(np.float32)).cuda()
        ref, got = _build_both(L, pts)
        # the build is deterministic, so the blobs match byte for byte
        assert torch.equal(ref, got)
        q = torch.from_numpy(rng.uniform(-3, 3, (4096, 3)).astype(np.float32)).cuda()
        np.testing.assert_array_equal(_query(L, got, pts, q), _query(L, ref, pts, q))


def test_noalloc_build_at_the_limit():
    """Exactly VT_BVH_NOALLOC_MAX_POINTS sites fit the fixed array."""
    from vorotracing_b200._lib import lib

    L = lib()
    n = 1_048_576
    rng = np.random.default_rng(1)
    pts = torch.from_numpy(rng.uniform(-2, 2, (n, 3)).astype(np.float32)).cuda()
    ref, got = _build_both(L, pts)
    assert torch.equal(ref, got)


def test_noalloc_rejects_too_many_sites():
    from vorotracing_b200._lib import lib

    L = lib()
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    st = L.vt_bvh_build_noalloc(C.c_void_p(dummy.data_ptr()), C.c_uint32(1_048_577),
                                C.c_void_p(dummy.data_ptr()), C.c_uint64(16), None)
    assert st == 1
    assert b"exceed the limit" in L.vt_last_error()
