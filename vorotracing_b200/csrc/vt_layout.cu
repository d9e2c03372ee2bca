// vt_layout.cu -- one-time scene and ray layout transforms of the inference
// path, as CUDA kernels (the reference does them with torch ops in Python).
//
//   vt_morton_codes     VoroTracingInfer._reorder_by_morton code computation
//                       (vorotracing/vorotracing.py:519-530): bbox-normalised
//                       10-bit-per-axis interleave, x bit i -> 3i, y -> 3i+1,
//                       z -> 3i+2, bbox extent clamped to >= 1e-6.
//   vt_morton_perm      perm = stable argsort(code) and its inverse (:532-534).
//                       The reference's torch.argsort is not stable; ties keep
//                       the original order here.
//   vt_gather_rows      dst[i] = src[perm[i]] for fixed-size rows (:536-543).
//   vt_permute_csr      new offsets = exclusive scan of counts[perm]; row i of
//                       the new CSR = row perm[i] of the old one with ids mapped
//                       through inv_perm, neighbour order kept (:545-570).
//   vt_tile_perm        the 4x8 warp-tile ray order of _tile_perm (:606-625),
//                       computed in closed form instead of by argsort.
//   vt_pad_f16x4        _pad_3to4 of a float32 map, rounding to binary16
//                       (RNE) as .half() does (:505-512).
//   vt_minmax_f32 / vt_quantize_u8   _quantize_to_uint8 (:495-503):
//                       q = clamp(rint((x - offset) / scale), 0, 255).
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "vt_abi.cuh"
#include "vt_geom.cuh"

namespace vt {
namespace layout {

__device__ __forceinline__ int f2ord(float f)
{
    int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff); }

__global__ void minmax_init(int *mm, int k)
{
    int t = threadIdx.x;
    if (t < k) {
        mm[2 * t] = 0x7fffffff;
        mm[2 * t + 1] = (int)0x80000000;
    }
}

// Column-wise min / max of a (rows, cols) float matrix, cols <= 4.
__global__ void minmax_kernel(const float *__restrict__ x, uint64_t rows, int cols, int *mm)
{
    float lo[4] = {3.4e38f, 3.4e38f, 3.4e38f, 3.4e38f};
    float hi[4] = {-3.4e38f, -3.4e38f, -3.4e38f, -3.4e38f};
    for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
         r += (uint64_t)gridDim.x * blockDim.x)
        for (int c = 0; c < cols; ++c) {
            float v = __ldg(x + r * cols + c);
            lo[c] = fminf(lo[c], v);
            hi[c] = fmaxf(hi[c], v);
        }
    for (int c = 0; c < cols; ++c) {
        for (int o = 16; o; o >>= 1) {
            lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
            hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
        }
        if ((threadIdx.x & 31) == 0) {
            atomicMin(mm + 2 * c, f2ord(lo[c]));
            atomicMax(mm + 2 * c + 1, f2ord(hi[c]));
        }
    }
}

__global__ void minmax_finish(const int *mm, int k, float *out)
{
    int t = threadIdx.x;
    if (t < 2 * k) out[t] = ord2f(mm[t]);
}

__global__ void morton_codes_kernel(const float *__restrict__ p, uint32_t n, const int *mm,
                                    int64_t *codes)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int64_t code = 0;
    int64_t q[3];
    for (int a = 0; a < 3; ++a) {
        float lo = ord2f(mm[2 * a]), hi = ord2f(mm[2 * a + 1]);
        float size = fmaxf(hi - lo, 1e-6f);
        float v = (__ldg(p + (size_t)i * 3 + a) - lo) / size * 1023.0f;
        v = fminf(fmaxf(v, 0.0f), 1023.0f);
        q[a] = (int64_t)v;
    }
    for (int b = 0; b < 10; ++b) {
        code |= ((q[0] >> b) & 1) << (3 * b);
        code |= ((q[1] >> b) & 1) << (3 * b + 1);
        code |= ((q[2] >> b) & 1) << (3 * b + 2);
    }
    codes[i] = code;
}

__global__ void iota_kernel(uint32_t *x, uint32_t n)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = i;
}

__global__ void narrow_codes(const int64_t *c64, uint32_t *c32, uint32_t n)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) c32[i] = (uint32_t)c64[i];
}

__global__ void invert_kernel(const uint32_t *perm, uint32_t *inv, uint32_t n)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) inv[perm[i]] = i;
}

__global__ void gather_rows_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                   const uint32_t *__restrict__ perm, uint32_t n, uint32_t row_bytes)
{
    // one warp per row; 16-byte moves when the row allows it
    uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    if (warp >= n) return;
    const uint8_t *s = src + (size_t)__ldg(perm + warp) * row_bytes;
    uint8_t *d = dst + (size_t)warp * row_bytes;
    if ((row_bytes & 15u) == 0 && ((uintptr_t)src & 15u) == 0 && ((uintptr_t)dst & 15u) == 0) {
        for (uint32_t k = lane; k < row_bytes / 16; k += 32)
            reinterpret_cast<uint4 *>(d)[k] = __ldg(reinterpret_cast<const uint4 *>(s) + k);
    } else if ((row_bytes & 3u) == 0 && ((uintptr_t)src & 3u) == 0 && ((uintptr_t)dst & 3u) == 0) {
        for (uint32_t k = lane; k < row_bytes / 4; k += 32)
            reinterpret_cast<uint32_t *>(d)[k] = __ldg(reinterpret_cast<const uint32_t *>(s) + k);
    } else {
        for (uint32_t k = lane; k < row_bytes; k += 32) d[k] = s[k];
    }
}

__global__ void counts_kernel(const uint32_t *offs, const uint32_t *perm, uint32_t n,
                              uint32_t *cnt)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        uint32_t c = perm[i];
        cnt[i] = offs[c + 1] - offs[c];
    }
    if (i == n) cnt[n] = 0;
}

__global__ void permute_csr_kernel(const uint32_t *__restrict__ offs,
                                   const uint32_t *__restrict__ adj,
                                   const uint32_t *__restrict__ perm,
                                   const uint32_t *__restrict__ inv,
                                   const uint32_t *__restrict__ new_offs, uint32_t n,
                                   uint32_t *__restrict__ new_adj)
{
    uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    if (warp >= n) return;
    uint32_t c = perm[warp];
    uint32_t b = offs[c], e = offs[c + 1];
    uint32_t nb = new_offs[warp];
    for (uint32_t k = lane; k < e - b; k += 32) new_adj[nb + k] = inv[adj[b + k]];
}

// Pixel traced by thread t for 4x8 tiles over an H x W image: tiles in row-major
// order, pixels row-major inside each tile, edge tiles clipped.  Equal to the
// argsort of the reference's key ((y//4)*ceil(W/8) + x//8)*32 + (y%4)*8 + x%8.
__global__ void tile_perm_kernel(uint32_t H, uint32_t W, uint32_t TH, uint32_t TW, uint32_t *out)
{
    uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)H * W) return;
    uint64_t band = (uint64_t)TH * W;
    uint32_t r = (uint32_t)(t / band);
    uint32_t local = (uint32_t)(t - (uint64_t)r * band);
    uint32_t hr = min(TH, H - r * TH);
    uint32_t tpr = (W + TW - 1) / TW;
    uint32_t c = min(local / (TW * hr), tpr - 1);
    uint32_t wc = min(TW, W - c * TW);
    uint32_t within = local - c * TW * hr;
    uint32_t yy = within / wc, xx = within % wc;
    out[t] = (r * TH + yy) * W + c * TW + xx;
}

__global__ void pad_f16x4_kernel(const float *__restrict__ src, uint64_t texels,
                                 uint2 *__restrict__ dst)
{
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= texels) return;
    const float *s = src + i * 3;
    uint2 o;
    o.x = (uint32_t)f2h(__ldg(s)) | ((uint32_t)f2h(__ldg(s + 1)) << 16);
    o.y = (uint32_t)f2h(__ldg(s + 2));
    dst[i] = o;
}

// (N*R^2 texels x 3 bytes) -> one 4-byte word per texel, 4th byte zero
__global__ void pad_u8x4_kernel(const uint8_t *__restrict__ src, uint64_t texels,
                                uint32_t *__restrict__ dst)
{
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= texels) return;
    const uint8_t *s = src + i * 3;
    dst[i] = (uint32_t)__ldg(s) | ((uint32_t)__ldg(s + 1) << 8) | ((uint32_t)__ldg(s + 2) << 16);
}

__global__ void quantize_kernel(const float *__restrict__ src, uint64_t count, float scale,
                                float offset, uint8_t *__restrict__ dst)
{
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float q = rintf((__ldg(src + i) - offset) / scale);
    q = fminf(fmaxf(q, 0.0f), 255.0f);
    dst[i] = (uint8_t)q;
}

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace layout
}  // namespace vt

using namespace vt::layout;

extern "C" vt_status vt_minmax_f32(const float *x, uint64_t rows, int cols, void *workspace,
                                   float *out, vt_stream stream)
{
    VT_REQUIRE(x && workspace && out && cols >= 1 && cols <= 4, "vt_minmax_f32: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;
    int *mm = (int *)workspace;
    minmax_init<<<1, 32, 0, s>>>(mm, cols);
    unsigned g = vt::grid_for(rows ? rows : 1, 256);
    minmax_kernel<<<g < 2368 ? g : 2368, 256, 0, s>>>(x, rows, cols, mm);
    minmax_finish<<<1, 32, 0, s>>>(mm, cols, out);
    return vt::check_launch("vt_minmax_f32");
}

extern "C" uint64_t vt_morton_workspace_bytes(uint32_t n)
{
    size_t sort_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (const uint32_t *)nullptr,
                                    (uint32_t *)nullptr, (const uint32_t *)nullptr,
                                    (uint32_t *)nullptr, (int)n, 0, 30);
    size_t scan_bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, (const uint32_t *)nullptr,
                                  (uint32_t *)nullptr, (int)n + 1);
    return 256 + 3 * a256((size_t)(n + 1) * 4) + a256(sort_bytes > scan_bytes ? sort_bytes
                                                                              : scan_bytes);
}

extern "C" vt_status vt_morton_codes(const float *points, uint32_t n, int64_t *codes,
                                     void *workspace, vt_stream stream)
{
    VT_REQUIRE(points && codes && workspace && n > 0, "vt_morton_codes: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;
    int *mm = (int *)workspace;
    minmax_init<<<1, 32, 0, s>>>(mm, 3);
    unsigned g = vt::grid_for(n, 256);
    minmax_kernel<<<g < 2368 ? g : 2368, 256, 0, s>>>(points, n, 3, mm);
    morton_codes_kernel<<<g, 256, 0, s>>>(points, n, mm, codes);
    return vt::check_launch("vt_morton_codes");
}

extern "C" vt_status vt_morton_perm(const int64_t *codes, uint32_t n, uint32_t *perm,
                                    uint32_t *inv_perm, void *workspace, uint64_t workspace_bytes,
                                    vt_stream stream)
{
    VT_REQUIRE(codes && perm && inv_perm && workspace && n > 0, "vt_morton_perm: bad arguments");
    VT_REQUIRE(workspace_bytes >= vt_morton_workspace_bytes(n), "vt_morton_perm: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    char *w = (char *)workspace + 256;
    uint32_t *c32 = (uint32_t *)w;  w += a256((size_t)(n + 1) * 4);
    uint32_t *c32o = (uint32_t *)w; w += a256((size_t)(n + 1) * 4);
    uint32_t *ids = (uint32_t *)w;  w += a256((size_t)(n + 1) * 4);
    size_t tb = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tb, c32, c32o, ids, perm, (int)n, 0, 30);
    unsigned g = vt::grid_for(n, 256);
    narrow_codes<<<g, 256, 0, s>>>(codes, c32, n);
    iota_kernel<<<g, 256, 0, s>>>(ids, n);
    cudaError_t e = cub::DeviceRadixSort::SortPairs(w, tb, c32, c32o, ids, perm, (int)n, 0, 30, s);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_morton_perm: %s", cudaGetErrorString(e));
    invert_kernel<<<g, 256, 0, s>>>(perm, inv_perm, n);
    return vt::check_launch("vt_morton_perm");
}

extern "C" vt_status vt_gather_rows(const void *src, void *dst, const uint32_t *perm, uint32_t n,
                                    uint32_t row_bytes, vt_stream stream)
{
    VT_REQUIRE(src && dst && perm && row_bytes > 0, "vt_gather_rows: bad arguments");
    if (n == 0) return VT_OK;
    gather_rows_kernel<<<vt::grid_for((uint64_t)n * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)src, (uint8_t *)dst, perm, n, row_bytes);
    return vt::check_launch("vt_gather_rows");
}

extern "C" vt_status vt_permute_csr(const uint32_t *offsets, const uint32_t *adjacency, uint32_t n,
                                    const uint32_t *perm, const uint32_t *inv_perm,
                                    uint32_t *new_offsets, uint32_t *new_adjacency,
                                    void *workspace, uint64_t workspace_bytes, vt_stream stream)
{
    VT_REQUIRE(offsets && adjacency && perm && inv_perm && new_offsets && new_adjacency &&
                   workspace && n > 0,
               "vt_permute_csr: bad arguments");
    VT_REQUIRE(workspace_bytes >= vt_morton_workspace_bytes(n), "vt_permute_csr: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    char *w = (char *)workspace + 256;
    uint32_t *cnt = (uint32_t *)w;
    w += 3 * a256((size_t)(n + 1) * 4);
    size_t tb = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, tb, cnt, new_offsets, (int)n + 1);
    counts_kernel<<<vt::grid_for(n + 1, 256), 256, 0, s>>>(offsets, perm, n, cnt);
    cudaError_t e = cub::DeviceScan::ExclusiveSum(w, tb, cnt, new_offsets, (int)n + 1, s);
    if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_permute_csr: %s", cudaGetErrorString(e));
    permute_csr_kernel<<<vt::grid_for((uint64_t)n * 32, 256), 256, 0, s>>>(
        offsets, adjacency, perm, inv_perm, new_offsets, n, new_adjacency);
    return vt::check_launch("vt_permute_csr");
}

extern "C" vt_status vt_tile_perm(uint32_t height, uint32_t width, uint32_t tile_h, uint32_t tile_w,
                                  uint32_t *perm, vt_stream stream)
{
    VT_REQUIRE(perm && tile_h > 0 && tile_w > 0, "vt_tile_perm: bad arguments");
    uint64_t n = (uint64_t)height * width;
    if (n == 0) return VT_OK;
    tile_perm_kernel<<<vt::grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(height, width, tile_h,
                                                                             tile_w, perm);
    return vt::check_launch("vt_tile_perm");
}

extern "C" vt_status vt_pad_f16x4(const float *src, uint64_t texels, void *dst, vt_stream stream)
{
    VT_REQUIRE(src && dst && ((uintptr_t)dst & 7u) == 0, "vt_pad_f16x4: bad arguments");
    if (texels == 0) return VT_OK;
    pad_f16x4_kernel<<<vt::grid_for(texels, 256), 256, 0, (cudaStream_t)stream>>>(src, texels,
                                                                                   (uint2 *)dst);
    return vt::check_launch("vt_pad_f16x4");
}

extern "C" vt_status vt_pad_u8x4(const uint8_t *src, uint64_t texels, void *dst, vt_stream stream)
{
    VT_REQUIRE(src && dst && ((uintptr_t)dst & 3u) == 0, "vt_pad_u8x4: bad arguments");
    if (texels == 0) return VT_OK;
    pad_u8x4_kernel<<<vt::grid_for(texels, 256), 256, 0, (cudaStream_t)stream>>>(src, texels,
                                                                                  (uint32_t *)dst);
    return vt::check_launch("vt_pad_u8x4");
}

extern "C" vt_status vt_quantize_u8(const float *src, uint64_t count, float scale, float offset,
                                    uint8_t *dst, vt_stream stream)
{
    VT_REQUIRE(src && dst, "vt_quantize_u8: bad arguments");
    if (count == 0) return VT_OK;
    quantize_kernel<<<vt::grid_for(count, 256), 256, 0, (cudaStream_t)stream>>>(src, count, scale,
                                                                                offset, dst);
    return vt::check_launch("vt_quantize_u8");
}
