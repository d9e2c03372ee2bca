"""Work partitioning across the GPUs of one box (one process per GPU).

Inference (no reference counterpart; the reference is single-GPU): the scene
is replicated and the independent units are views (``view_shard``) or, for a
single large frame, interleaved bands of 4 pixel rows, the height of a 4x8
warp tile (``row_band_shard``).  Neither needs a collective on the data path.

Training: every rank renders its own rays against the same scene, and the
per-cell gradients are summed across ranks with one NCCL all-reduce of a
flat fp32 bucket [points 3N | density N | diffuse 3R^2 N | specular 3R^2 N]
(``GradBucket``).  The backward kernel writes straight into views of the
bucket, so the reduction needs no packing copy.  ``GradBucket.allreduce_``
is that reduction with NCCL; ``PeerGradReducer`` fuses it with the
backward's compaction pass in one kernel over peer memory (CUDA IPC,
NVLink): each rank reads its slice of every rank's backward workspace, sums
in rank order and writes the result into every rank's bucket.
"""
from __future__ import annotations

import numpy as np
import torch


def view_shard(n_views: int, rank: int, world: int) -> list[int]:
    """Views of this rank, round-robin."""
    return list(range(rank, n_views, world))


def row_band_shard(height: int, rank: int, world: int, band: int = 4) -> np.ndarray:
    """Pixel rows of this rank: bands of ``band`` rows dealt round-robin."""
    rows = np.arange(height)
    return rows[(rows // band) % world == rank]


class GradBucket:
    """Flat gradient buffer with per-parameter views laid out for one all-reduce."""

    def __init__(self, n_points: int, tex_cols: int, device, dtype=torch.float32):
        self.n = n_points
        self.tex_cols = tex_cols
        sizes = [3 * n_points, n_points, tex_cols * n_points, tex_cols * n_points]
        self.flat = torch.zeros(sum(sizes), dtype=dtype, device=device)
        parts = torch.split(self.flat, sizes)
        self.points = parts[0].view(n_points, 3)
        self.density = parts[1].view(n_points, 1)
        self.diffuse = parts[2].view(n_points, tex_cols)
        self.specular = parts[3].view(n_points, tex_cols)

    def views(self):
        return self.points, self.diffuse, self.specular, self.density

    def zero_(self):
        self.flat.zero_()
        return self

    def allreduce_(self, group=None, average: bool = False):
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            if average:
                self.flat.div_(dist.get_world_size(group))
        return self

    @property
    def nbytes(self) -> int:
        return self.flat.numel() * self.flat.element_size()


class PeerGradReducer:
    """All-reduce of a GradBucket fused with the backward's compaction, over
    the peer memory of the ranks of one node (vt_grad_allreduce_peer).

    Every rank allocates its backward workspace and a staging buffer here
    and maps the other ranks' buckets and staging buffers (CUDA IPC handles
    exchanged through the process group).  A step is

        trace_vorotracing_bwd(..., grads=bucket.views(), accumulate=False,
                              workspace=red.workspace, keep_workspace=True)
        red.reduce_()

    ``reduce_`` runs phase 0 (this rank's compacted shares stored into their
    owners' staging buffers), a fence, phase 1 (this rank's share summed in
    rank order and stored into every bucket) and a fence.  The fences are
    one-element all-reduces of the process group, stream-ordered: every
    rank's phase 0 before any phase 1, every phase 1 before the buckets are
    read and the staging buffers written again.  The kernels never wait on
    another GPU.  fp32 attributes only."""

    def __init__(self, bucket: GradBucket, res: int, group=None):
        import ctypes as C

        import torch.distributed as dist

        from . import _lib

        self.bucket = bucket
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.PEER_MAX:
            raise RuntimeError(f"PeerGradReducer: at most {_lib.PEER_MAX} ranks")
        if bucket.flat.dtype != torch.float32:
            raise RuntimeError("PeerGradReducer: fp32 buckets only")
        L = _lib.lib()
        dev = bucket.flat.device
        wsb = int(L.vt_trace_bwd_workspace_bytes(C.c_uint32(bucket.n), C.c_int(res)))
        slot = int(L.vt_peer_staging_floats(C.c_uint32(bucket.n), C.c_int(res),
                                            C.c_uint32(self.world)))
        self.workspace = torch.empty(wsb, dtype=torch.uint8, device=dev)
        self.staging = torch.empty(self.world * slot, dtype=torch.float32, device=dev)
        mine = []
        for t in (bucket.flat, self.staging):
            h = (C.c_uint8 * 64)()
            off = C.c_uint64(0)
            _lib.check(L.vt_ipc_handle(C.c_void_p(t.data_ptr()), h, C.byref(off)), "vt_ipc_handle")
            mine.append((bytes(h), int(off.value)))
        table = [None] * self.world
        dist.all_gather_object(table, mine, group=group)
        self._opened = []
        g = _lib.VtPeerGrads()
        g.world, g.num_points, g.res = self.world, bucket.n, res
        g.workspace[self.rank] = self.workspace.data_ptr()
        try:
            for k in range(self.world):
                if k == self.rank:
                    b_p, s_p = bucket.flat.data_ptr(), self.staging.data_ptr()
                else:
                    ptrs = []
                    for handle, off in table[k]:
                        base = C.c_void_p()
                        _lib.check(L.vt_ipc_open((C.c_uint8 * 64).from_buffer_copy(handle),
                                                 C.byref(base)), "vt_ipc_open")
                        self._opened.append(base.value)
                        ptrs.append(base.value + off)
                    b_p, s_p = ptrs
                g.bucket[k] = b_p
                g.staging[k] = s_p
        except RuntimeError:
            for base in self._opened:  # unmap what was mapped before the failure
                L.vt_ipc_close(C.c_void_p(base))
            self._opened = []
            raise
        self._args = g
        self._fence = torch.zeros(1, dtype=torch.int32, device=dev)

    def reduce_(self):
        import ctypes as C

        import torch.distributed as dist

        from . import _lib

        L = _lib.lib()
        stream = _lib.stream_ptr(self.bucket.flat.device)
        _lib.check(L.vt_grad_allreduce_peer(C.byref(self._args), C.c_uint32(self.rank),
                                            C.c_uint32(0), stream), "vt_grad_allreduce_peer")
        dist.all_reduce(self._fence, group=self.group)
        _lib.check(L.vt_grad_allreduce_peer(C.byref(self._args), C.c_uint32(self.rank),
                                            C.c_uint32(1), stream), "vt_grad_allreduce_peer")
        dist.all_reduce(self._fence, group=self.group)
        return self.bucket

    def close(self):
        import ctypes as C

        from . import _lib

        torch.cuda.synchronize()
        for base in self._opened:
            _lib.lib().vt_ipc_close(C.c_void_p(base))
        self._opened = []
