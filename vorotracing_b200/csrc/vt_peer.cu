// vt_peer.cu -- the training step's gradient all-reduce over peer memory.
//
// After the backward (vt_trace_bwd with VT_BWD_KEEP_WORKSPACE) every rank
// holds its texel and site gradient sums in its padded fp32 workspace (one
// float4 per texel / site) and its density gradients in its flat bucket.
// The reference trains on one GPU; here the replacement for "compact the
// workspace into the bucket, then all-reduce the bucket with NCCL" is one
// kernel per rank: rank r owns a 1/world slice of every array, reads that
// slice from all ranks' workspaces and buckets (peer loads over NVLink), sums
// in rank order, drops the padding and writes the result into the slice of
// every rank's bucket (peer stores).  The workspace bytes cross NVLink once
// and the local compaction pass disappears.  Slices are disjoint, so no two
// ranks write the same words; ordering with the backward and with the next
// step is the caller's (stream-ordered fences), and the kernel itself never
// waits on another GPU.
#include <cstring>

#include "vt_abi.cuh"

namespace vt {
namespace {

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

struct PeerArgs {
    uint32_t world;
    const float4 *sdiff[VT_PEER_MAX];
    const float4 *sspec[VT_PEER_MAX];
    const float4 *spts[VT_PEER_MAX];
    float *bucket[VT_PEER_MAX];
    uint64_t n, ntex;
    uint64_t begin, end;  // this rank's slice of the combined item space
};

// Item space: [0, ntex) diffuse texels, [ntex, 2 ntex) specular texels,
// [2 ntex, 2 ntex + n) sites, [2 ntex + n, 2 ntex + 2 n) densities.
template <int W>
__global__ void __launch_bounds__(256) peer_reduce_kernel(PeerArgs a)
{
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t n = a.n, ntex = a.ntex;
    const uint32_t world = W > 0 ? (uint32_t)W : a.world;
    for (uint64_t it = a.begin + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < a.end;
         it += stride) {
        if (it < 2 * ntex + n) {
            const float4 *const *src;
            uint64_t i, out;
            if (it < ntex) {
                src = a.sdiff;
                i = it;
                out = 4 * n + 3 * i;
            } else if (it < 2 * ntex) {
                src = a.sspec;
                i = it - ntex;
                out = 4 * n + 3 * ntex + 3 * i;
            } else {
                src = a.spts;
                i = it - 2 * ntex;
                out = 3 * i;
            }
            float4 acc = __ldcs(src[0] + i);
            for (uint32_t k = 1; k < world; ++k) {
                const float4 v = __ldcs(src[k] + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
            }
            for (uint32_t k = 0; k < world; ++k) {
                float *o = a.bucket[k] + out;
                o[0] = acc.x;
                o[1] = acc.y;
                o[2] = acc.z;
            }
        } else {
            const uint64_t i = 3 * n + (it - 2 * ntex - n);
            float acc = __ldcs(a.bucket[0] + i);
            for (uint32_t k = 1; k < world; ++k) acc += __ldcs(a.bucket[k] + i);
            for (uint32_t k = 0; k < world; ++k) a.bucket[k][i] = acc;
        }
    }
    // make the peer stores visible before the caller's fence
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

extern "C" vt_status vt_grad_allreduce_peer(const vt_peer_grads *g, uint32_t rank,
                                            vt_stream stream)
{
    VT_REQUIRE(g, "vt_grad_allreduce_peer: null argument");
    VT_REQUIRE(g->world >= 1 && g->world <= VT_PEER_MAX, "vt_grad_allreduce_peer: world %u out of range",
               g->world);
    VT_REQUIRE(rank < g->world, "vt_grad_allreduce_peer: rank %u >= world %u", rank, g->world);
    VT_REQUIRE(g->res == 4 || g->res == 8, "vt_grad_allreduce_peer: res must be 4 or 8");
    VT_REQUIRE(g->num_points > 0, "vt_grad_allreduce_peer: no points");
    vt::PeerArgs a{};
    a.world = g->world;
    a.n = g->num_points;
    a.ntex = (uint64_t)g->num_points * g->res * g->res;
    for (uint32_t k = 0; k < g->world; ++k) {
        VT_REQUIRE(g->workspace[k] && g->bucket[k], "vt_grad_allreduce_peer: rank %u buffers missing", k);
        VT_REQUIRE((((uintptr_t)g->workspace[k]) & 255u) == 0 && (((uintptr_t)g->bucket[k]) & 3u) == 0,
                   "vt_grad_allreduce_peer: workspace must be 256-byte aligned");
        const char *w = (const char *)g->workspace[k];
        a.sdiff[k] = (const float4 *)w;
        a.sspec[k] = (const float4 *)(w + vt::a256(a.ntex * 16));
        a.spts[k] = (const float4 *)(w + 2 * vt::a256(a.ntex * 16));
        a.bucket[k] = g->bucket[k];
    }
    const uint64_t total = 2 * a.ntex + 2 * a.n;
    const uint64_t share = (total + g->world - 1) / g->world;
    a.begin = share * rank;
    a.end = a.begin + share < total ? a.begin + share : total;
    if (a.begin >= a.end) return VT_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t want = (a.end - a.begin + 255) / 256;
    const unsigned grid = (unsigned)(want < (uint64_t)sms * 8 ? want : (uint64_t)sms * 8);
    cudaStream_t s = (cudaStream_t)stream;
    switch (g->world) {
    case 2: vt::peer_reduce_kernel<2><<<grid, 256, 0, s>>>(a); break;
    case 4: vt::peer_reduce_kernel<4><<<grid, 256, 0, s>>>(a); break;
    case 8: vt::peer_reduce_kernel<8><<<grid, 256, 0, s>>>(a); break;
    default: vt::peer_reduce_kernel<0><<<grid, 256, 0, s>>>(a); break;
    }
    return vt::check_launch("peer_reduce_kernel");
}
