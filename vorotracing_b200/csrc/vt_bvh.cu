// vt_bvh.cu -- nearest-site BVH for the ray-origin cell lookup.
//
// Replaces the reference's cuBQL binary BVH and findClosest query
// (vorotracing/cuda/csrc/utils/nn_bvh.cu:12-117).  Build: 30-bit Morton
// codes of the sites, a stable radix sort of (code, id), Karras' (HPG 2012)
// parallel construction of the binary radix tree (codes are disambiguated by
// their sorted position), and a bottom-up box pass in which the second child
// to arrive at a node computes its box (an atomic counter, no waiting).
// Query: depth-first, nearest child first, pruning subtrees whose box is
// strictly farther than the best site so far.
//
// Exact contract (matches the CPU oracle's brute force): the answer minimises
// d2 = fma(dz,dz, fma(dy,dy, dx*dx)) in binary32, ties to the lowest site index.
// The box bound is computed with the same rounded operations, and RN is
// monotone, so a box bound never exceeds the d2 of any site inside it.
//
// Blob layout written by vt_bvh_build (vt_bvh_nodes_bytes(n) bytes):
//   Node nodes[n-1]   internal nodes (32 B: box + two child links)
//   uint32 ids[n]     site id of each leaf (sorted order)
// A child link with bit 31 set names leaf (link & 0x7fffffff).
#include <cub/device/device_radix_sort.cuh>

#include "vt_abi.cuh"
#include "vt_bvh.cuh"

namespace vt {
namespace bvh {


__device__ __forceinline__ int f2ord(float f)
{
    int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff); }

__global__ void bbox_init(int *bb)
{
    if (threadIdx.x < 3) bb[threadIdx.x] = 0x7fffffff;
    else if (threadIdx.x < 6) bb[threadIdx.x] = (int)0x80000000;
}

__global__ void bbox_kernel(const float *__restrict__ p, uint32_t n, int *bb)
{
    float lo[3] = {3.4e38f, 3.4e38f, 3.4e38f}, hi[3] = {-3.4e38f, -3.4e38f, -3.4e38f};
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        for (int a = 0; a < 3; ++a) {
            float v = __ldg(p + (size_t)i * 3 + a);
            lo[a] = fminf(lo[a], v);
            hi[a] = fmaxf(hi[a], v);
        }
    for (int a = 0; a < 3; ++a)
        for (int o = 16; o; o >>= 1) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    if ((threadIdx.x & 31) == 0)
        for (int a = 0; a < 3; ++a) {
            atomicMin(bb + a, f2ord(lo[a]));
            atomicMax(bb + 3 + a, f2ord(hi[a]));
        }
}

__device__ __forceinline__ uint32_t spread10(uint32_t v)
{
    v &= 0x3ffu;
    v = (v | (v << 16)) & 0x030000ffu;
    v = (v | (v << 8)) & 0x0300f00fu;
    v = (v | (v << 4)) & 0x030c30c3u;
    v = (v | (v << 2)) & 0x09249249u;
    return v;
}

__global__ void morton_kernel(const float *__restrict__ p, uint32_t n, const int *bb,
                              uint32_t *codes, uint32_t *ids)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t c = 0;
    for (int a = 0; a < 3; ++a) {
        float lo = ord2f(bb[a]), hi = ord2f(bb[3 + a]);
        float ext = fmaxf(hi - lo, 1e-20f);
        float x = (__ldg(p + (size_t)i * 3 + a) - lo) / ext * 1023.0f;
        uint32_t q = (uint32_t)fminf(fmaxf(x, 0.0f), 1023.0f);
        c |= spread10(q) << a;
    }
    codes[i] = c;
    ids[i] = i;
}

__device__ __forceinline__ int delta(const uint32_t *codes, int n, int i, int j)
{
    if (j < 0 || j >= n) return -1;
    uint32_t a = codes[i], b = codes[j];
    if (a == b) return 32 + __clz((uint32_t)i ^ (uint32_t)j);
    return __clz(a ^ b);
}

__global__ void karras_kernel(const uint32_t *__restrict__ codes, int n, Node *nodes,
                              uint32_t *parent_int, uint32_t *parent_leaf, uint32_t *flags)
{
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n - 1) return;
    int d = (delta(codes, n, i, i + 1) - delta(codes, n, i, i - 1)) >= 0 ? 1 : -1;
    int dmin = delta(codes, n, i, i - d);
    int lmax = 2;
    while (delta(codes, n, i, i + lmax * d) > dmin) lmax <<= 1;
    int l = 0;
    for (int t = lmax >> 1; t >= 1; t >>= 1)
        if (delta(codes, n, i, i + (l + t) * d) > dmin) l += t;
    int j = i + l * d;
    int dnode = delta(codes, n, i, j);
    int s = 0;
    for (int div = 2;; div <<= 1) {
        int t = (l + div - 1) / div;
        if (delta(codes, n, i, i + (s + t) * d) > dnode) s += t;
        if (t == 1) break;
    }
    int g = i + s * d + (d < 0 ? -1 : 0);
    int lo = min(i, j), hi = max(i, j);
    uint32_t left = (lo == g) ? (kLeaf | (uint32_t)g) : (uint32_t)g;
    uint32_t right = (hi == g + 1) ? (kLeaf | (uint32_t)(g + 1)) : (uint32_t)(g + 1);
    nodes[i].left = left;
    nodes[i].right = right;
    if (left & kLeaf) parent_leaf[g] = i; else parent_int[g] = i;
    if (right & kLeaf) parent_leaf[g + 1] = i; else parent_int[g + 1] = i;
    flags[i] = 0;
}

__device__ __forceinline__ void child_box(const Node *nodes, const uint32_t *ids,
                                          const float *p, uint32_t link, float lo[3], float hi[3])
{
    if (link & kLeaf) {
        const float *q = p + (size_t)ids[link & ~kLeaf] * 3;
        for (int a = 0; a < 3; ++a) lo[a] = hi[a] = q[a];
    } else {
        volatile const Node *c = nodes + link;
        for (int a = 0; a < 3; ++a) {
            lo[a] = c->lo[a];
            hi[a] = c->hi[a];
        }
    }
}

__global__ void boxes_kernel(const float *__restrict__ p, int n, Node *nodes,
                             const uint32_t *__restrict__ ids, const uint32_t *parent_int,
                             const uint32_t *parent_leaf, uint32_t *flags)
{
    int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    uint32_t node = parent_leaf[k];
    for (int guard = 0; guard < 2 * n; ++guard) {
        __threadfence();
        if (atomicAdd(flags + node, 1u) == 0) return;  // first child: the sibling finishes
        float la[3], ha[3], lb[3], hb[3];
        child_box(nodes, ids, p, nodes[node].left, la, ha);
        child_box(nodes, ids, p, nodes[node].right, lb, hb);
        for (int a = 0; a < 3; ++a) {
            nodes[node].lo[a] = fminf(la[a], lb[a]);
            nodes[node].hi[a] = fmaxf(ha[a], hb[a]);
        }
        if (node == 0) return;
        node = parent_int[node];
    }
}


__device__ __forceinline__ void visit_leaf(const float *__restrict__ p, uint32_t id, V3 q,
                                           float &best, uint32_t &bi)
{
    V3 d = q - ld3(p + (size_t)id * 3);
    float d2 = dot(d, d);
    if (d2 < best || (d2 == best && id < bi)) {
        best = d2;
        bi = id;
    }
}

// A hint (a site believed nearest, e.g. the answer for a neighbouring query)
// only seeds the bound: the result is the same lexicographic (d2, id) minimum,
// found with tighter pruning when the hint is good.
// Depth-first search from the root for one query: nearest child first,
// subtrees pruned when their bound exceeds the best d2 so far.
__device__ __forceinline__ void query_thread(const Node *__restrict__ nodes,
                                             const uint32_t *__restrict__ ids,
                                             const float *__restrict__ p, V3 q, float &best,
                                             uint32_t &bi, uint32_t *err)
{
    uint32_t stack[kStack];
    int sp = 0;
    uint32_t cur = 0;
    for (;;) {
        if (cur & kLeaf) {
            visit_leaf(p, __ldg(ids + (cur & ~kLeaf)), q, best, bi);
        } else {
            const Node nd = nodes[cur];
            uint32_t c[2] = {nd.left, nd.right};
            float dd[2];
            for (int k = 0; k < 2; ++k) {
                if (c[k] & kLeaf) {
                    V3 dv = q - ld3(p + (size_t)__ldg(ids + (c[k] & ~kLeaf)) * 3);
                    dd[k] = dot(dv, dv);
                } else {
                    dd[k] = box_d2(nodes[c[k]], q);
                }
            }
            int nearf = dd[1] < dd[0] ? 1 : 0;
            bool go_near = dd[nearf] <= best;
            bool go_far = dd[1 - nearf] <= best;
            if (go_far) {
                if (sp >= kStack) {
                    report(err, VT_ERR_DATA);
                    break;
                }
                stack[sp++] = c[1 - nearf];
            }
            if (go_near) {
                cur = c[nearf];
                continue;
            }
        }
        // pop the next subtree that can still hold a closer (or equal, lower id) site
        bool found = false;
        while (sp > 0) {
            uint32_t s = stack[--sp];
            float dd;
            if (s & kLeaf) {
                V3 dv = q - ld3(p + (size_t)__ldg(ids + (s & ~kLeaf)) * 3);
                dd = dot(dv, dv);
            } else {
                dd = box_d2(nodes[s], q);
            }
            if (dd <= best) {
                cur = s;
                found = true;
                break;
            }
        }
        if (!found) break;
    }
}

// A hint (a site believed nearest, e.g. the answer for a neighbouring query)
// only seeds the bound: the result is the same lexicographic (d2, id) minimum,
// found with tighter pruning when the hint is good.
__global__ void query_kernel(const Node *__restrict__ nodes, const uint32_t *__restrict__ ids,
                             const float *__restrict__ p, uint32_t n,
                             const float *__restrict__ queries, uint32_t nq,
                             const uint32_t *__restrict__ hint, uint32_t hint_count, int32_t *out,
                             uint32_t *err)
{
    uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nq) return;
    V3 q = mk(__ldg(queries + (size_t)t * 3), __ldg(queries + (size_t)t * 3 + 1),
              __ldg(queries + (size_t)t * 3 + 2));
    float best = __int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu;
    if (hint) {
        const uint32_t h = __ldg(hint + (hint_count == 1 ? 0 : t));
        if (h < n) visit_leaf(p, h, q, best, bi);
    }
    if (n == 1)
        visit_leaf(p, 0, q, best, bi);
    else
        query_thread(nodes, ids, p, q, best, bi, err);
    out[t] = (int32_t)bi;
}

// Warp-cooperative query (packet traversal).  The 32 lanes of a warp hold 32
// queries, in the callers' order neighbouring ray origins, and, when they are
// close together (see below), walk the tree together: one warp-uniform current node and one warp-wide stack (entry k in
// register k / 32 of lane k % 32, popped by a shuffle).  A child is entered
// when any lane's bound admits it (ballot), nearer child first by lane vote,
// and a leaf child is visited at once.  Node and site loads are warp-uniform
// (one broadcast transaction) and no lane diverges from the traversal.  Each
// lane still prunes with its own bound, so its answer is the same
// lexicographic (d2, id) minimum as query_kernel's: the warp visits a
// superset of the subtrees each lane needs.  Lanes past nq take part with an
// empty bound (best < 0 admits nothing).
__global__ void __launch_bounds__(128) query_warp_kernel(
    const Node *__restrict__ nodes, const uint32_t *__restrict__ ids, const float *__restrict__ p,
    uint32_t n, const float *__restrict__ queries, uint32_t nq, const uint32_t *__restrict__ hint,
    uint32_t hint_count, int32_t *out, uint32_t *err)
{
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t lane = threadIdx.x & 31u;
    const bool valid = t < nq;
    V3 q = mk(0.f, 0.f, 0.f);
    float best = -1.0f;
    uint32_t bi = 0xffffffffu;
    if (valid) {
        q = mk(__ldg(queries + (size_t)t * 3), __ldg(queries + (size_t)t * 3 + 1),
               __ldg(queries + (size_t)t * 3 + 2));
        best = __int_as_float(0x7f800000);
        if (hint) {
            const uint32_t h = __ldg(hint + (hint_count == 1 ? 0 : t));
            if (h < n) visit_leaf(p, h, q, best, bi);
        }
    }
    if (__ballot_sync(0xffffffffu, valid) == 0) return;
    if (n == 1) {
        if (valid) {
            visit_leaf(p, 0, q, best, bi);
            out[t] = (int32_t)bi;
        }
        return;
    }
    // The warp traverses together only when its queries are close compared
    // with the typical distance between sites, s = (scene box volume / n)^(1/3),
    // the scale of a nearest-site search ball: the squared diagonal of the
    // queries' box at most 16 s^2.  The lanes' search balls then overlap and
    // their union is little more than one.  Otherwise every lane searches on
    // its own (a warp of scattered queries would visit the union of all their
    // searches).
    float lo[3] = {q.x, q.y, q.z}, hi[3] = {q.x, q.y, q.z};
    if (!valid) {
        lo[0] = lo[1] = lo[2] = __int_as_float(0x7f800000);
        hi[0] = hi[1] = hi[2] = __int_as_float(0xff800000);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    }
    const V3 ext = mk(hi[0] - lo[0], hi[1] - lo[1], hi[2] - lo[2]);
    const float diag2 = dot(ext, ext);
    const Node root = nodes[0];
    const float vol = fmaxf((root.hi[0] - root.lo[0]) * (root.hi[1] - root.lo[1]) *
                                (root.hi[2] - root.lo[2]),
                            0.0f);
    const float spacing = cbrtf(vol / (float)n);
    const bool packet = diag2 <= 16.0f * spacing * spacing;
    if (!packet) {
        if (valid) {
            query_thread(nodes, ids, p, q, best, bi, err);
            out[t] = (int32_t)bi;
        }
        return;
    }
    uint32_t st0 = 0, st1 = 0, st2 = 0;  // the warp's stack, distributed over the lanes
    int sp = 0;
    uint32_t cur = 0;
    bool overflow = false;
    for (;;) {
        // cur is an internal node here
        const Node nd = nodes[cur];
        const uint32_t c[2] = {nd.left, nd.right};
        float dd[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (c[k] & kLeaf) {
                const uint32_t id = __ldg(ids + (c[k] & ~kLeaf));
                if (valid) visit_leaf(p, id, q, best, bi);
                dd[k] = __int_as_float(0x7f800000);  // visited: nothing left below
            } else {
                dd[k] = valid ? box_d2(nodes[c[k]], q) : __int_as_float(0x7f800000);
            }
        }
        const bool need0 = __any_sync(0xffffffffu, dd[0] <= best);
        const bool need1 = __any_sync(0xffffffffu, dd[1] <= best);
        if (need0 && need1) {
            const int votes1 = __popc(__ballot_sync(0xffffffffu, valid && dd[1] < dd[0]));
            const int votes0 = __popc(__ballot_sync(0xffffffffu, valid && dd[0] < dd[1]));
            const int nearc = votes1 > votes0 ? 1 : 0;
            if (sp >= 3 * 32) {
                overflow = true;
                break;
            }
            const uint32_t far = c[1 - nearc];
            if ((uint32_t)(sp & 31) == lane) {
                if (sp < 32) st0 = far;
                else if (sp < 64) st1 = far;
                else st2 = far;
            }
            sp++;
            cur = c[nearc];
            continue;
        }
        if (need0) {
            cur = c[0];
            continue;
        }
        if (need1) {
            cur = c[1];
            continue;
        }
        // pop the next subtree that any lane can still improve in
        bool found = false;
        while (sp > 0) {
            --sp;
            const uint32_t reg = sp < 32 ? st0 : (sp < 64 ? st1 : st2);
            const uint32_t sub = __shfl_sync(0xffffffffu, reg, sp & 31);
            const float d = valid ? box_d2(nodes[sub], q) : __int_as_float(0x7f800000);
            if (__any_sync(0xffffffffu, d <= best)) {
                cur = sub;
                found = true;
                break;
            }
        }
        if (!found) break;
    }
    if (overflow && lane == 0) report(err, VT_ERR_DATA);
    if (valid) out[t] = (int32_t)bi;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Scratch of the radix sort.  If cub's size query fails, an upper bound is
// returned instead of its (then undefined) answer: the sort's alternate key
// and value buffers plus 1 MiB for its histograms, so a workspace sized from
// this value is never too small.
size_t sort_temp_bytes(uint32_t n)
{
    size_t bytes = 0;
    cudaError_t e = cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint32_t *)nullptr,
                                                    (uint32_t *)nullptr, (const uint32_t *)nullptr,
                                                    (uint32_t *)nullptr, (int)n, 0, 30);
    if (e != cudaSuccess) return (size_t)n * 8 + (size_t(1) << 20);
    return bytes;
}

}  // namespace bvh
}  // namespace vt

using vt::bvh::align256;
using vt::bvh::Node;

// Batches of at least this many queries use the warp-cooperative traversal
// (building with -DVT_WARP_QUERY_MIN=0xffffffff keeps every batch per-thread).
#ifndef VT_WARP_QUERY_MIN
#define VT_WARP_QUERY_MIN 32
#endif
static constexpr uint32_t kWarpQueryMin = VT_WARP_QUERY_MIN;

extern "C" uint64_t vt_bvh_nodes_bytes(uint32_t num_points)
{
    return align256((size_t)(num_points ? num_points - 1 : 0) * sizeof(Node)) +
           (size_t)num_points * 4;
}

extern "C" uint64_t vt_bvh_workspace_bytes(uint32_t n)
{
    return 256 + 4 * align256((size_t)n * 4) + 3 * align256((size_t)n * 4) +
           align256(vt::bvh::sort_temp_bytes(n));
}

extern "C" vt_status vt_bvh_build(const float *points, uint32_t num_points, void *nodes,
                                  uint64_t nodes_bytes, void *workspace, uint64_t workspace_bytes,
                                  vt_stream stream)
{
    VT_REQUIRE(points && nodes && workspace, "vt_bvh_build: null pointer");
    VT_REQUIRE(num_points > 0 && num_points < 0x7fffffffu, "vt_bvh_build: bad point count");
    VT_REQUIRE(nodes_bytes >= vt_bvh_nodes_bytes(num_points), "vt_bvh_build: nodes buffer too small");
    VT_REQUIRE(workspace_bytes >= vt_bvh_workspace_bytes(num_points),
               "vt_bvh_build: workspace too small");
    VT_REQUIRE(((uintptr_t)nodes & 255u) == 0 && ((uintptr_t)workspace & 255u) == 0,
               "vt_bvh_build: buffers must be 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    const uint32_t n = num_points;
    char *w = (char *)workspace;
    int *bb = (int *)w;
    w += 256;
    uint32_t *codes_in = (uint32_t *)w;  w += align256((size_t)n * 4);
    uint32_t *codes_out = (uint32_t *)w; w += align256((size_t)n * 4);
    uint32_t *ids_in = (uint32_t *)w;    w += align256((size_t)n * 4);
    uint32_t *parent_leaf = (uint32_t *)w; w += align256((size_t)n * 4);
    uint32_t *parent_int = (uint32_t *)w;  w += align256((size_t)n * 4);
    uint32_t *flags = (uint32_t *)w;       w += align256((size_t)n * 4);
    w += align256((size_t)n * 4);  // reserved (keeps the workspace layout of vt_bvh_workspace_bytes)
    size_t temp_bytes = vt::bvh::sort_temp_bytes(n);
    void *temp = w;
    Node *nd = (Node *)nodes;
    uint32_t *ids = (uint32_t *)((char *)nodes + align256((size_t)(n - 1) * sizeof(Node)));

    vt::bvh::bbox_init<<<1, 32, 0, s>>>(bb);
    unsigned g = vt::grid_for(n, 256);
    vt::bvh::bbox_kernel<<<g < 1184 ? g : 1184, 256, 0, s>>>(points, n, bb);
    vt::bvh::morton_kernel<<<g, 256, 0, s>>>(points, n, bb, codes_in, ids_in);
    cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, codes_in, codes_out, ids_in,
                                                    ids, (int)n, 0, 30, s);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_bvh_build sort: %s", cudaGetErrorString(e));
    if (n > 1) {
        vt::bvh::karras_kernel<<<vt::grid_for(n - 1, 256), 256, 0, s>>>(codes_out, (int)n, nd,
                                                                         parent_int, parent_leaf, flags);
        vt::bvh::boxes_kernel<<<g, 256, 0, s>>>(points, (int)n, nd, ids, parent_int, parent_leaf,
                                                flags);
    }
    return vt::check_launch("vt_bvh_build");
}

extern "C" vt_status vt_bvh_query(const void *nodes, const float *points, uint32_t num_points,
                                  const float *queries, uint32_t num_queries, int32_t *out,
                                  uint32_t *err, vt_stream stream)
{
    VT_REQUIRE(nodes && points && num_points > 0, "vt_bvh_query: BVH must be built before querying");
    VT_REQUIRE(num_queries == 0 || (queries && out), "vt_bvh_query: null query buffers");
    if (num_queries == 0) return VT_OK;
    const Node *nd = (const Node *)nodes;
    const uint32_t *ids =
        (const uint32_t *)((const char *)nodes + align256((size_t)(num_points - 1) * sizeof(Node)));
    if (num_queries >= kWarpQueryMin)
        vt::bvh::query_warp_kernel<<<vt::grid_for(num_queries, 128), 128, 0,
                                     (cudaStream_t)stream>>>(nd, ids, points, num_points, queries,
                                                             num_queries, nullptr, 0, out, err);
    else
        vt::bvh::query_kernel<<<vt::grid_for(num_queries, 128), 128, 0, (cudaStream_t)stream>>>(
            nd, ids, points, num_points, queries, num_queries, nullptr, 0, out, err);
    return vt::check_launch("vt_bvh_query");
}

extern "C" vt_status vt_bvh_query_hint(const void *nodes, const float *points, uint32_t num_points,
                                       const float *queries, uint32_t num_queries,
                                       const uint32_t *hint, uint32_t hint_count, int32_t *out,
                                       uint32_t *err, vt_stream stream)
{
    VT_REQUIRE(nodes && points && num_points > 0,
               "vt_bvh_query_hint: BVH must be built before querying");
    VT_REQUIRE(num_queries == 0 || (queries && out), "vt_bvh_query_hint: null query buffers");
    VT_REQUIRE(hint && (hint_count == 1 || hint_count == num_queries),
               "vt_bvh_query_hint: hint must hold 1 or num_queries site ids");
    if (num_queries == 0) return VT_OK;
    const Node *nd = (const Node *)nodes;
    const uint32_t *ids =
        (const uint32_t *)((const char *)nodes + align256((size_t)(num_points - 1) * sizeof(Node)));
    if (num_queries >= kWarpQueryMin)
        vt::bvh::query_warp_kernel<<<vt::grid_for(num_queries, 128), 128, 0,
                                     (cudaStream_t)stream>>>(nd, ids, points, num_points, queries,
                                                             num_queries, hint, hint_count, out,
                                                             err);
    else
        vt::bvh::query_kernel<<<vt::grid_for(num_queries, 128), 128, 0, (cudaStream_t)stream>>>(
            nd, ids, points, num_points, queries, num_queries, hint, hint_count, out, err);
    return vt::check_launch("vt_bvh_query_hint");
}

// ---------------------------------------------------------------------------
// Allocation-free BVH build.
//
// Some callers cannot allocate device memory themselves: a host application
// that hands this library only its input and output buffers and keeps every
// other byte of device memory under its own budget, or a binding whose
// language runtime has no CUDA allocator to offer.  vt_bvh_build_noalloc
// gives them the start-cell BVH build with its scratch in a fixed array that
// lives in this file (kNoAllocScratchBytes on every GPU that loads the
// library, held until the process exits).  Sites are limited to
// VT_BVH_NOALLOC_MAX_POINTS.
//
// Host code cannot pass the array's name to a kernel: on the host that name
// is only a stand-in symbol, not a device address.  The first call on each
// device resolves the device address with cudaGetSymbolAddress (with that
// device current) and caches it; make that first call before any stream
// capture.  All calls share the one array, so calls whose work overlaps on
// the GPU (different streams, or different host threads on one device) race
// on it; serialise them.  The cached address belongs to the device's primary
// context: after cudaDeviceReset (or anything else that destroys that
// context) this library must be unloaded and loaded again before the next
// call.  The array keeps the previous call's contents: every
// field the build reads (bounding box, sort buffers, parent links, the
// per-node arrival counters) is rewritten by the build before it is read.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

// vt_bvh_workspace_bytes(VT_BVH_NOALLOC_MAX_POINTS) is 28 MiB + 256 B of
// build buffers plus the radix sort's scratch, which holds alternate key and
// value buffers (8 MiB) and its histograms: 40 MiB covers it with room to
// spare (the build checks the exact need on every call).
constexpr size_t kNoAllocScratchBytes = size_t(40) << 20;
static __device__ __align__(256) unsigned char g_bvh_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[256] = {};

}  // namespace

extern "C" vt_status vt_bvh_build_noalloc(const float *points, uint32_t num_points, void *nodes,
                                          uint64_t nodes_bytes, vt_stream stream)
{
    VT_REQUIRE(num_points <= VT_BVH_NOALLOC_MAX_POINTS,
               "vt_bvh_build_noalloc: %u sites exceed the limit of %u for the fixed scratch "
               "array; use vt_bvh_build with a caller-provided workspace",
               num_points, (unsigned)VT_BVH_NOALLOC_MAX_POINTS);
    const uint64_t need = vt_bvh_workspace_bytes(num_points);
    VT_REQUIRE(need <= kNoAllocScratchBytes,
               "vt_bvh_build_noalloc: %llu scratch bytes needed, %llu available",
               (unsigned long long)need, (unsigned long long)kNoAllocScratchBytes);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return vt::set_error(VT_ERR_CUDA, "vt_bvh_build_noalloc: %s", cudaGetErrorString(e));
    VT_REQUIRE(dev >= 0 && dev < 256, "vt_bvh_build_noalloc: device index %d out of range", dev);
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_bvh_noalloc_scratch);
            if (e != cudaSuccess)
                return vt::set_error(VT_ERR_CUDA, "vt_bvh_build_noalloc: cudaGetSymbolAddress: %s",
                                     cudaGetErrorString(e));
            g_noalloc_ptr[dev] = p;
        }
        scratch = g_noalloc_ptr[dev];
    }
    return vt_bvh_build(points, num_points, nodes, nodes_bytes, scratch, kNoAllocScratchBytes,
                        stream);
}
