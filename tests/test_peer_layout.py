"""Host-side layout of the peer all-reduce (no GPU needed): the staging
slot from vt_peer_staging_floats holds every rank's share of the bucket, the
shares tile the bucket in the GradBucket order, and bad arguments give 0."""
import ctypes as C

import pytest


def _share_floats(n, res, world):
    """Floats of each rank's contiguous share of the bucket [points 3n |
    density n | diffuse 3R^2 n | specular 3R^2 n], items in bucket order."""
    ntex = n * res * res

    def off(i):
        if i < n:
            return 3 * i
        if i < 2 * n:
            return 3 * n + (i - n)
        return 4 * n + 3 * (i - 2 * n)

    total = 2 * n + 2 * ntex
    share = -(-total // world)
    out = []
    for r in range(world):
        b, e = min(total, share * r), min(total, share * (r + 1))
        out.append(off(e) - off(b))
    return out


@pytest.mark.parametrize("n,res,world", [(1, 4, 1), (5, 4, 3), (1000, 8, 2), (3_000_000, 8, 8),
                                         (17, 8, 7)])
def test_staging_slot_covers_every_share(n, res, world):
    from vorotracing_b200 import _lib
    from vorotracing_b200.shard import GradBucket

    L = _lib.lib()
    slot = int(L.vt_peer_staging_floats(C.c_uint32(n), C.c_int(res), C.c_uint32(world)))
    shares = _share_floats(n, res, world)
    assert slot % 64 == 0 and slot >= max(shares)
    assert slot - max(shares) < 64
    # the shares tile the whole bucket
    cols = 3 * res * res
    assert sum(shares) == 3 * n + n + 2 * cols * n
    if n < 2000:
        b = GradBucket(n, cols, "cpu")
        assert b.flat.numel() == sum(shares)


def test_staging_floats_rejects_bad_arguments():
    from vorotracing_b200 import _lib

    L = _lib.lib()
    assert L.vt_peer_staging_floats(C.c_uint32(10), C.c_int(8), C.c_uint32(0)) == 0
    assert L.vt_peer_staging_floats(C.c_uint32(0), C.c_int(8), C.c_uint32(2)) == 0
    assert L.vt_peer_staging_floats(C.c_uint32(10), C.c_int(5), C.c_uint32(2)) == 0
