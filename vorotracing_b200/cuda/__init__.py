"""Drop-in replacement for the reference's ``vorotracing.cuda`` operator module
(vorotracing/cuda/__init__.py:49-57): same names, argument meaning, tensor
layouts and error behaviour, backed by the sm_100a kernels of
libvorotracing_b200.so."""
from ._ops import NNBVH, build_voronoi_adjacency, nearest_neighbor_bvh
from ._wrapper import (
    ErrorBox,
    TraceVoroTracing,
    prefetch_octmap_adj,
    trace_octmap_infer,
    trace_octmap_infer_q8,
)

__all__ = [
    "TraceVoroTracing",
    "trace_octmap_infer",
    "trace_octmap_infer_q8",
    "prefetch_octmap_adj",
    "build_voronoi_adjacency",
    "NNBVH",
    "nearest_neighbor_bvh",
]
