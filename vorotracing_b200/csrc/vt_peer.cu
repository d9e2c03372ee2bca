// vt_peer.cu -- the training step's gradient all-reduce over peer memory.
//
// After the backward (vt_trace_bwd with VT_BWD_KEEP_WORKSPACE) every rank
// holds its texel and site gradient sums in its padded fp32 workspace (one
// float4 per texel / site) and its density gradients in its flat bucket.
// The reference trains on one GPU; here "compact the workspace into the
// bucket, then all-reduce the bucket with NCCL" becomes two kernels per rank
// over peer memory, every cross-GPU access a posted store:
//   phase 0  rank r compacts its workspace (drops the float4 padding) and
//            writes each other rank's share of the result into slot r of
//            that rank's staging buffer (a reduce-scatter by stores);
//   phase 1  rank r sums its own share over the ranks in rank order (its
//            workspace and the staging slots) and writes the sums into that
//            share of every rank's bucket (an all-gather by stores).
// NVLink carries (world-1)/world of the compact bucket twice, the bytes of
// an ideal all-reduce, and the local compaction pass is folded into phase
// 0.  Shares are disjoint, so no two ranks write the same words.  Ordering
// (every phase 0 before any phase 1, every phase 1 before the next use) is
// the caller's, with stream-ordered fences; the kernels never wait on
// another GPU.
#include <cstring>

#include "vt_abi.cuh"

namespace vt {
namespace {

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// Items in bucket order: sites [0, n), densities [n, 2n), diffuse texels
// [2n, 2n + ntex), specular texels [2n + ntex, 2n + 2 ntex).  Item i's
// floats in the bucket start at bucket_off(i) (3 per site or texel, 1 per
// density), so a contiguous item range is a contiguous bucket range.
struct Layout {
    uint64_t n, ntex;
    __host__ __device__ uint64_t bucket_off(uint64_t i) const
    {
        if (i < n) return 3 * i;
        if (i < 2 * n) return 3 * n + (i - n);
        return 4 * n + 3 * (i - 2 * n);
    }
    __host__ __device__ uint64_t items() const { return 2 * n + 2 * ntex; }
};

struct PeerArgs {
    uint32_t world, rank;
    Layout L;
    uint64_t share;                 // items per rank (the last rank may own fewer)
    uint64_t slot;                  // floats per staging slot
    const float4 *sdiff, *sspec, *spts;  // this rank's workspace
    float *bucket[VT_PEER_MAX];
    float *staging[VT_PEER_MAX];
};

// This rank's compacted value of item i: up to 3 floats (1 for a density).
__device__ __forceinline__ int local_item(const PeerArgs &a, uint64_t i, float v[3])
{
    const uint64_t n = a.L.n, ntex = a.L.ntex;
    if (i >= n && i < 2 * n) {
        v[0] = __ldcs(a.bucket[a.rank] + 3 * n + (i - n));
        return 1;
    }
    const float4 q = i < n ? __ldcs(a.spts + i)
                           : (i < 2 * n + ntex ? __ldcs(a.sdiff + (i - 2 * n))
                                               : __ldcs(a.sspec + (i - 2 * n - ntex)));
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    return 3;
}

// Phase 0: every item outside this rank's share goes, compacted, into slot
// `rank` of its owner's staging buffer.
__global__ void __launch_bounds__(256) peer_push_kernel(PeerArgs a)
{
    const uint64_t total = a.L.items();
    const uint64_t mine_b = a.share * a.rank, mine_e = min(total, mine_b + a.share);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        if (i >= mine_b && i < mine_e) continue;
        const uint32_t owner = (uint32_t)(i / a.share);
        float v[3] = {0.f, 0.f, 0.f};
        const int c = local_item(a, i, v);
        float *dst = a.staging[owner] + (uint64_t)a.rank * a.slot +
                     (a.L.bucket_off(i) - a.L.bucket_off(a.share * owner));
        dst[0] = v[0];
        if (c == 3) {
            dst[1] = v[1];
            dst[2] = v[2];
        }
    }
    __threadfence_system();
}

// Phase 1: this rank's share, summed in rank order, into every bucket.
__global__ void __launch_bounds__(256) peer_reduce_kernel(PeerArgs a)
{
    const uint64_t total = a.L.items();
    const uint64_t b = a.share * a.rank, e = min(total, b + a.share);
    const uint64_t base = a.L.bucket_off(b);
    const float *stage = a.staging[a.rank];
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = b + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += stride) {
        const uint64_t off = a.L.bucket_off(i), rel = off - base;
        float mine[3] = {0.f, 0.f, 0.f};
        const int c = local_item(a, i, mine);
        float acc[3] = {0.f, 0.f, 0.f};
        for (uint32_t k = 0; k < a.world; ++k) {
            float v[3] = {0.f, 0.f, 0.f};
            if (k == a.rank) {
                v[0] = mine[0];
                v[1] = mine[1];
                v[2] = mine[2];
            } else {
                const float *src = stage + (uint64_t)k * a.slot + rel;
                v[0] = __ldcs(src);
                if (c == 3) {
                    v[1] = __ldcs(src + 1);
                    v[2] = __ldcs(src + 2);
                }
            }
            if (k == 0) {
                acc[0] = v[0];
                acc[1] = v[1];
                acc[2] = v[2];
            } else {
                acc[0] += v[0];
                if (c == 3) {
                    acc[1] += v[1];
                    acc[2] += v[2];
                }
            }
        }
        for (uint32_t k = 0; k < a.world; ++k) {
            float *o = a.bucket[k] + off;
            o[0] = acc[0];
            if (c == 3) {
                o[1] = acc[1];
                o[2] = acc[2];
            }
        }
    }
    __threadfence_system();
}

}  // namespace
}  // namespace vt

extern "C" vt_status vt_ipc_handle(const void *ptr, void *handle64, uint64_t *offset)
{
    VT_REQUIRE(ptr && handle64 && offset, "vt_ipc_handle: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    // the allocation's base address, from the driver (looked up through the
    // runtime so that the library does not link libcuda)
    typedef int (*range_fn)(unsigned long long *, size_t *, unsigned long long);
    static range_fn get_range = nullptr;
    if (!get_range) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return vt::set_error(VT_ERR_CUDA, "vt_ipc_handle: cuMemGetAddressRange unavailable");
        get_range = (range_fn)fn;
    }
    unsigned long long b = 0;
    size_t size = 0;
    const int r = get_range(&b, &size, (unsigned long long)(uintptr_t)ptr);
    if (r != 0) return vt::set_error(VT_ERR_CUDA, "vt_ipc_handle: address range query failed (%d)", r);
    void *base = (void *)(uintptr_t)b;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, base);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_ipc_handle: %s", cudaGetErrorString(e));
    memcpy(handle64, &h, sizeof(h));
    *offset = (uint64_t)((const char *)ptr - (const char *)base);
    return VT_OK;
}

extern "C" vt_status vt_ipc_open(const void *handle64, void **base)
{
    VT_REQUIRE(handle64 && base, "vt_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_ipc_open: %s", cudaGetErrorString(e));
    return VT_OK;
}

extern "C" vt_status vt_ipc_close(void *base)
{
    VT_REQUIRE(base, "vt_ipc_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_ipc_close: %s", cudaGetErrorString(e));
    return VT_OK;
}

extern "C" uint64_t vt_peer_staging_floats(uint32_t num_points, int res, uint32_t world)
{
    if (world == 0 || num_points == 0 || (res != 4 && res != 8)) return 0;
    const vt::Layout L{num_points, (uint64_t)num_points * res * res};
    const uint64_t total = L.items(), share = (total + world - 1) / world;
    uint64_t m = 0;
    for (uint32_t r = 0; r < world; ++r) {
        const uint64_t b = share * r < total ? share * r : total;
        const uint64_t e = b + share < total ? b + share : total;
        const uint64_t f = (e == total ? 4 * L.n + 6 * L.ntex : L.bucket_off(e)) - L.bucket_off(b);
        m = f > m ? f : m;
    }
    return (m + 63) & ~(uint64_t)63;  // 256-byte aligned slots
}

extern "C" vt_status vt_grad_allreduce_peer(const vt_peer_grads *g, uint32_t rank, uint32_t phase,
                                            vt_stream stream)
{
    VT_REQUIRE(g, "vt_grad_allreduce_peer: null argument");
    VT_REQUIRE(g->world >= 1 && g->world <= VT_PEER_MAX, "vt_grad_allreduce_peer: world %u out of range",
               g->world);
    VT_REQUIRE(rank < g->world, "vt_grad_allreduce_peer: rank %u >= world %u", rank, g->world);
    VT_REQUIRE(phase <= 1, "vt_grad_allreduce_peer: phase must be 0 or 1");
    VT_REQUIRE(g->res == 4 || g->res == 8, "vt_grad_allreduce_peer: res must be 4 or 8");
    VT_REQUIRE(g->num_points > 0, "vt_grad_allreduce_peer: no points");
    for (uint32_t k = 0; k < g->world; ++k)
        VT_REQUIRE(g->bucket[k] && g->staging[k], "vt_grad_allreduce_peer: rank %u buffers missing", k);
    VT_REQUIRE(g->workspace[rank] && (((uintptr_t)g->workspace[rank]) & 255u) == 0,
               "vt_grad_allreduce_peer: the workspace must be 256-byte aligned");
    vt::PeerArgs a{};
    a.world = g->world;
    a.rank = rank;
    a.L = vt::Layout{g->num_points, (uint64_t)g->num_points * g->res * g->res};
    a.share = (a.L.items() + g->world - 1) / g->world;
    a.slot = vt_peer_staging_floats(g->num_points, g->res, g->world);
    const char *w = (const char *)g->workspace[rank];
    a.sdiff = (const float4 *)w;
    a.sspec = (const float4 *)(w + vt::a256(a.L.ntex * 16));
    a.spts = (const float4 *)(w + 2 * vt::a256(a.L.ntex * 16));
    for (uint32_t k = 0; k < g->world; ++k) {
        a.bucket[k] = g->bucket[k];
        a.staging[k] = g->staging[k];
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t items = phase == 0 ? a.L.items() : a.share;
    const uint64_t want = (items + 255) / 256;
    const unsigned grid = (unsigned)(want < (uint64_t)sms * 8 ? (want ? want : 1) : (uint64_t)sms * 8);
    cudaStream_t s = (cudaStream_t)stream;
    if (phase == 0) {
        if (g->world > 1) vt::peer_push_kernel<<<grid, 256, 0, s>>>(a);
    } else {
        vt::peer_reduce_kernel<<<grid, 256, 0, s>>>(a);
    }
    return vt::check_launch("vt_grad_allreduce_peer");
}
