// vt_pack.cu -- packed face rows (replaces prefetch_adjacent_diff_octmap_kernel,
// tracing_octmap.cu:125-149, and its host wrapper :612-640).  The same pass
// can also write the reference's own (adjacency_len + 32, 4) binary16 rows,
// which callers of the reference's operator keep and export.
//
// One warp per cell, lanes over the cell's CSR row, so reads of the adjacency
// row and the 16-byte record stores are coalesced (the reference uses one
// thread per cell with a serial loop and 8-byte scattered stores).  The kernel
// also validates the CSR it packs: neighbour ids < N, monotone offsets and
// degrees that fit the record's 16-bit field; violations set *err.
#include "vt_abi.cuh"
#include "vt_geom.cuh"

namespace vt {

__global__ void __launch_bounds__(256) pack_faces_kernel(
    const float *__restrict__ points, uint32_t n, const uint32_t *__restrict__ adj,
    const uint32_t *__restrict__ offs, uint64_t csr_entries, uint4 *__restrict__ faces,
    uint64_t rows, uint2 *__restrict__ diff4, uint64_t diff_rows, uint32_t *err)
{
    const uint64_t gtid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t r = csr_entries + gtid; r < rows; r += nthreads) faces[r] = make_uint4(0, 0, 0, 0);
    if (diff4)
        for (uint64_t r = csr_entries + gtid; r < diff_rows; r += nthreads)
            diff4[r] = make_uint2(0, 0);

    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warp = gtid >> 5;
    const uint64_t nwarps = nthreads >> 5;
    for (uint64_t cell = warp; cell < n; cell += nwarps) {
        uint32_t b = __ldg(offs + cell), e = __ldg(offs + cell + 1);
        if (e < b || e > csr_entries) {
            if (lane == 0) report(err, VT_ERR_DATA);
            continue;
        }
        V3 P = ld3(points + cell * 3);
        for (uint32_t k = b + lane; k < e; k += 32) {
            uint32_t nb = __ldg(adj + k);
            if (nb >= n) {
                report(err, VT_ERR_DATA);
                faces[k] = make_uint4(0, 0, 0, 0);
                if (diff4) diff4[k] = make_uint2(0, 0);
                continue;
            }
            V3 Q = ld3(points + (size_t)nb * 3);
            uint32_t nbeg = __ldg(offs + nb);
            uint32_t ndeg = __ldg(offs + nb + 1) - nbeg;
            if (ndeg > kMaxDegree) {
                report(err, VT_ERR_DATA);
                ndeg = 0;
            }
            V3 d = Q - P;
            uint4 f;
            f.x = (uint32_t)f2h(d.x) | ((uint32_t)f2h(d.y) << 16);
            f.y = (uint32_t)f2h(d.z) | (ndeg << 16);
            f.z = nb;
            f.w = nbeg;
            faces[k] = f;
            // the reference's half4 row: the same three binary16 differences, zero w
            if (diff4) diff4[k] = make_uint2(f.x, f.y & 0xffffu);
        }
    }
}

}  // namespace vt

extern "C" uint64_t vt_face_rows(uint64_t csr_entries) { return csr_entries + vt::kFacePadRows; }

extern "C" vt_status vt_prefetch_adj(const float *points, uint32_t num_points,
                                     const uint32_t *adjacency, uint64_t adjacency_len,
                                     const uint32_t *offsets, uint64_t csr_entries, void *faces,
                                     uint64_t face_rows, uint32_t *err, vt_stream stream)
{
    VT_REQUIRE(points && offsets && faces, "vt_prefetch_adj: null pointer");
    VT_REQUIRE(num_points > 0, "vt_prefetch_adj: num_points must be > 0");
    VT_REQUIRE(csr_entries == 0 || adjacency, "vt_prefetch_adj: null adjacency");
    VT_REQUIRE(csr_entries <= adjacency_len,
               "vt_prefetch_adj: offsets[N] = %llu exceeds adjacency length %llu",
               (unsigned long long)csr_entries, (unsigned long long)adjacency_len);
    VT_REQUIRE(face_rows >= vt_face_rows(csr_entries), "vt_prefetch_adj: faces buffer too small");
    VT_REQUIRE(((uintptr_t)faces & 15u) == 0, "vt_prefetch_adj: faces must be 16-byte aligned");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    uint64_t want = ((uint64_t)num_points * 32 + 255) / 256;
    unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? (want ? want : 1) : (uint64_t)sms * 16);
    vt::pack_faces_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        points, num_points, adjacency, offsets, csr_entries, (uint4 *)faces, face_rows, nullptr, 0,
        err);
    return vt::check_launch("pack_faces_kernel");
}

extern "C" uint64_t vt_adj_diff_rows(uint64_t adjacency_len) { return adjacency_len + 32; }

extern "C" vt_status vt_prefetch_adj_diff(const float *points, uint32_t num_points,
                                          const uint32_t *adjacency, uint64_t adjacency_len,
                                          const uint32_t *offsets, uint64_t csr_entries,
                                          void *faces, uint64_t face_rows, void *adj_diff,
                                          uint64_t adj_diff_rows, uint32_t *err, vt_stream stream)
{
    VT_REQUIRE(points && offsets && faces && adj_diff, "vt_prefetch_adj_diff: null pointer");
    VT_REQUIRE(num_points > 0, "vt_prefetch_adj_diff: num_points must be > 0");
    VT_REQUIRE(csr_entries == 0 || adjacency, "vt_prefetch_adj_diff: null adjacency");
    VT_REQUIRE(csr_entries <= adjacency_len,
               "vt_prefetch_adj_diff: offsets[N] = %llu exceeds adjacency length %llu",
               (unsigned long long)csr_entries, (unsigned long long)adjacency_len);
    VT_REQUIRE(face_rows >= vt_face_rows(csr_entries), "vt_prefetch_adj_diff: faces buffer too small");
    VT_REQUIRE(adj_diff_rows >= csr_entries, "vt_prefetch_adj_diff: adj_diff buffer too small");
    VT_REQUIRE(((uintptr_t)faces & 15u) == 0 && ((uintptr_t)adj_diff & 7u) == 0,
               "vt_prefetch_adj_diff: faces must be 16-byte and adj_diff 8-byte aligned");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    uint64_t want = ((uint64_t)num_points * 32 + 255) / 256;
    unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? (want ? want : 1) : (uint64_t)sms * 16);
    vt::pack_faces_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        points, num_points, adjacency, offsets, csr_entries, (uint4 *)faces, face_rows,
        (uint2 *)adj_diff, adj_diff_rows, err);
    return vt::check_launch("pack_faces_kernel");
}
