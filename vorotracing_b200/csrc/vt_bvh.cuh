// vt_bvh.cuh -- node layout of the nearest-site BVH (built by vt_bvh.cu) and
// the box distance bound its traversals prune with.
//
// Blob layout written by vt_bvh_build (vt_bvh_nodes_bytes(n) bytes):
//   Node nodes[n-1]   internal nodes (32 B: box + two child links), root = 0
//   uint32 ids[n]     site id of each leaf (sorted order), 256-byte aligned
// A child link with bit 31 set names leaf (link & 0x7fffffff).
#pragma once

#include "vt_geom.cuh"

namespace vt {
namespace bvh {

struct __align__(16) Node {
    float lo[3];
    uint32_t left;
    float hi[3];
    uint32_t right;
};

constexpr uint32_t kLeaf = 0x80000000u;
constexpr int kStack = 96;

__device__ __forceinline__ float box_d2(const Node &b, V3 q)
{
    float dx = fmaxf(fmaxf(b.lo[0] - q.x, 0.0f), q.x - b.hi[0]);
    float dy = fmaxf(fmaxf(b.lo[1] - q.y, 0.0f), q.y - b.hi[1]);
    float dz = fmaxf(fmaxf(b.lo[2] - q.z, 0.0f), q.z - b.hi[2]);
    // same contracted form as the site distance dot(d, d), so the bound stays
    // below the distance of every site in the box (RN and fma are monotone)
    return dot(mk(dx, dy, dz), mk(dx, dy, dz));
}

// Leaf ids follow the nodes at the next 256-byte boundary.
__host__ __device__ inline const uint32_t *leaf_ids(const void *blob, uint32_t n)
{
    const size_t nb = ((size_t)(n ? n - 1 : 0) * sizeof(Node) + 255) & ~(size_t)255;
    return (const uint32_t *)((const char *)blob + nb);
}

}  // namespace bvh
}  // namespace vt
