/*
 * vorotracing_b200.h -- C ABI of the B200-native Voronoi ray-traversal library
 * (libvorotracing_b200.so).
 *
 * Plain pointers and sizes only.  Every pointer named *device* is CUDA global
 * memory on the current device; every call is asynchronous on `stream`
 * (0 = legacy default stream) and allocates nothing: outputs and scratch are
 * passed in by the caller, scratch sizes come from the *_bytes queries.
 * Calls return VT_OK or an error code; vt_last_error() returns the message
 * of the last failure on the calling thread.  Errors found by kernels in the
 * data (bad CSR, degree overflow, start index out of range) are written to
 * the optional device word `err` as a vt_status and become visible after the
 * stream is synchronised.
 *
 * Reference interfaces replaced (paths inside the VoroTracing project):
 *   vt_prefetch_adj        trace_vorotracing_prefetch_adj, vorotracing/cuda/csrc/tracing/tracing_octmap.h:33-36
 *   vt_prefetch_adj_diff   the same, also writing its (E+32, 4) half4 output, tracing_octmap.cu:612-640
 *   vt_trace_infer_f16     trace_vorotracing_infer,        tracing_octmap.h:38-51
 *   vt_trace_infer_q8      trace_vorotracing_infer_q8,     tracing_octmap.h:53-67
 *   vt_trace_fwd           trace_vorotracing_fwd,          tracing_octmap.h:11-31
 *   vt_trace_bwd           trace_vorotracing_bwd,          tracing_octmap.h:69-91
 *   vt_bvh_build/query     NNBVH::build / NNBVH::query,    vorotracing/cuda/csrc/utils/nn_bvh.h:4-18
 *   vt_morton_*, vt_permute_csr      VoroTracingInfer._reorder_by_morton, vorotracing/vorotracing.py:514-571
 *   vt_tile_perm           VoroTracingInfer._tile_perm,    vorotracing.py:606-625
 *   vt_pad_f16x4           VoroTracingInfer._pad_3to4,     vorotracing.py:505-512
 *   vt_minmax_f32, vt_quantize_u8    VoroTracingInfer._quantize_to_uint8, vorotracing.py:495-503
 */
#ifndef VOROTRACING_B200_H
#define VOROTRACING_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VT_API __attribute__((visibility("default")))
#else
#define VT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int vt_status;
#define VT_OK 0
#define VT_ERR_INVALID 1 /* bad argument (null pointer, size, alignment) */
#define VT_ERR_CUDA 2    /* CUDA runtime error */
#define VT_ERR_DATA 3    /* inconsistent scene data found by a kernel */

typedef struct CUstream_st *vt_stream; /* == cudaStream_t */

/* Message of the last failed call on this thread ("" if none). */
VT_API const char *vt_last_error(void);
/* Library version, e.g. "0.1.0". */
VT_API const char *vt_version(void);
/* Device address of page-locked host memory (cudaHostAlloc / cudaHostRegister
 * with mapping; every such allocation is mapped under unified addressing).
 * The trace entry points accept it for rays and rgba, so that a kernel reads
 * its rays from and writes its pixels to host memory over the bus while it
 * runs (zero-copy end-to-end render).  No reference counterpart: the
 * reference's operators take device tensors only. */
VT_API vt_status vt_host_device_ptr(const void *host, void **device);

/* Scene in device memory.  points (N,3) f32, density (N) f32, offsets (N+1)
 * u32 CSR, faces = packed face rows written by vt_prefetch_adj. */
typedef struct {
    const float *points;
    const float *density;
    const uint32_t *offsets;
    const void *faces;
    uint32_t num_points;
    uint64_t num_face_rows;
} vt_scene;

/* Optional per-ray diagnostics (any field may be null). */
typedef struct {
    uint32_t *seq;               /* (rays, seq_cap) visited cell ids */
    uint32_t seq_cap;
    uint32_t *seq_len;           /* (rays) cells visited */
    uint32_t *stats;             /* (rays, 4) steps, faces tested, segments, textured */
    uint32_t *num_intersections; /* (rays) walk step count as the reference returns it */
    uint8_t *visited;            /* (N) set to 1 for every cell a ray visits */
    uint8_t *textured;           /* (N) set to 1 for every cell whose texels are read */
} vt_debug;

/* ---- packed faces (replaces the reference's adj_diff half4 rows) ---- */

/* Rows of 16 bytes needed for a CSR with `csr_entries` = offsets[N] entries. */
VT_API uint64_t vt_face_rows(uint64_t csr_entries);
/* Build the packed face rows: per CSR entry e of cell i, half(points[adj[e]] -
 * points[i]), the neighbour id, its CSR begin and its degree.  csr_entries =
 * offsets[N] (read on the host by the caller). */
VT_API vt_status vt_prefetch_adj(const float *points, uint32_t num_points, const uint32_t *adjacency,
                          uint64_t adjacency_len, const uint32_t *offsets, uint64_t csr_entries,
                          void *faces, uint64_t face_rows, uint32_t *err, vt_stream stream);
/* Rows of the reference's adj_diff for an adjacency array of adjacency_len
 * entries: adjacency_len + 32 (tracing_octmap.cu:624-625). */
VT_API uint64_t vt_adj_diff_rows(uint64_t adjacency_len);
/* vt_prefetch_adj plus, in the same pass, the reference's adj_diff array
 * (trace_vorotracing_prefetch_adj, tracing_octmap.cu:612-640): adj_diff_rows
 * rows of four binary16, half(points[adj[e]] - points[i]) and 0 for CSR entry
 * e of cell i, zero rows after offsets[N].  adj_diff 8-byte aligned. */
VT_API vt_status vt_prefetch_adj_diff(const float *points, uint32_t num_points,
                                      const uint32_t *adjacency, uint64_t adjacency_len,
                                      const uint32_t *offsets, uint64_t csr_entries, void *faces,
                                      uint64_t face_rows, void *adj_diff, uint64_t adj_diff_rows,
                                      uint32_t *err, vt_stream stream);

/* ---- inference ---- */

/* fp16 inference.  diffuse/specular: (N, 4*res*res) binary16 (Half4Texel:
 * rgb + zero pad).  rays (num_rays, 6) f32, 8-byte aligned.  start (num_rays)
 * u32.  ray_perm (num_rays) u32 or null (thread t traces ray ray_perm[t]).
 * rgba (num_rays, 4) binary16 out, in ray order.  res = 4 or 8. */
VT_API vt_status vt_trace_infer_f16(const vt_scene *scene, const void *diffuse, const void *specular,
                             int res, const float *rays, uint32_t num_rays, const uint32_t *start,
                             const uint32_t *ray_perm, float weight_threshold,
                             uint32_t max_intersections, float cell_skip_threshold, void *rgba,
                             const vt_debug *debug, uint32_t *err, vt_stream stream);

/* q8 inference.  diffuse/specular (N, 3*res*res) u8 with one global scale and
 * offset per map: value = scale * q + offset. */
VT_API vt_status vt_trace_infer_q8(const vt_scene *scene, const uint8_t *diffuse, const uint8_t *specular,
                            int res, float diff_scale, float diff_offset, float spec_scale,
                            float spec_offset, const float *rays, uint32_t num_rays,
                            const uint32_t *start, const uint32_t *ray_perm,
                            float weight_threshold, uint32_t max_intersections,
                            float cell_skip_threshold, void *rgba, const vt_debug *debug,
                            uint32_t *err, vt_stream stream);
/* vt_trace_infer_q8 on texels widened to 4 bytes (r, g, b, 0; vt_pad_u8x4):
 * diffuse/specular (N, 4*res*res) u8, 4-byte aligned.  Same pixels, one
 * 32-bit load per texel instead of three byte loads.  No reference
 * counterpart (an internal layout of the reference's q8 maps). */
VT_API vt_status vt_trace_infer_q8x4(const vt_scene *scene, const void *diffuse,
                                     const void *specular, int res, float diff_scale,
                                     float diff_offset, float spec_scale, float spec_offset,
                                     const float *rays, uint32_t num_rays, const uint32_t *start,
                                     const uint32_t *ray_perm, float weight_threshold,
                                     uint32_t max_intersections, float cell_skip_threshold,
                                     void *rgba, const vt_debug *debug, uint32_t *err,
                                     vt_stream stream);

/* Depth render (the viewer's depth modes, vorotracing/viewer.py:414-433; no
 * kernel counterpart in the reference, which runs the full training forward
 * with a per-ray copy of the thresholds).  thresholds: K transmittance
 * levels shared by all rays, decreasing, device memory.  Training-forward
 * transmittance rule, no colour.  depth (num_rays) f32 out, in ray order:
 * VT_DEPTH_FIRST_QUANTILE the depth where T falls below thresholds[0];
 * VT_DEPTH_MEAN the mean of the positive quantile depths; -1 where none. */
#define VT_DEPTH_FIRST_QUANTILE 0
#define VT_DEPTH_MEAN 1
VT_API vt_status vt_trace_depth(const vt_scene *scene, const float *rays, uint32_t num_rays,
                                const uint32_t *start, const uint32_t *ray_perm,
                                const float *thresholds, uint32_t num_thresholds, int mode,
                                float weight_threshold, uint32_t max_intersections,
                                float *depth, uint32_t *err, vt_stream stream);

/* ---- training ---- */

/* Path record: the training forward stores, for each ray and walk step, the
 * cell it enters and the colour it computed for the segment integrated at
 * that step: steps (cap, num_rays) records of 16 bytes {u32 cell, f32 r, g,
 * b} (0 colour for untextured cells and empty segments), slot-major:
 * steps[k * num_rays + r], 16-byte aligned; len (num_rays) u32 = the number
 * of steps that found an exit face (steps beyond cap are not stored).  Bit 31
 * of len flags a ray that the backward must walk itself: the record
 * overflowed, or the forward stopped at T == weight_threshold exactly (the
 * backward's stop rule is T < weight_threshold).  Given the same record, the
 * backward enters the recorded cells of the other rays without scanning their
 * faces and without re-reading their texels, and walks the flagged ones in a
 * second launch (replaying their stored prefix first), with results identical
 * to a backward without the record.  The record is only valid for the inputs
 * of the forward that wrote it.  No reference counterpart (the reference's
 * backward re-walks every ray). */
typedef struct {
    void *steps;
    uint32_t cap;
    uint32_t *len;
} vt_path;

/* Training forward (attr_half = 0: f32 attributes and rgba; 1: binary16).
 * diffuse/specular (N, 3*res*res).  depth_quantiles (num_rays, K) f32 or null
 * (K = 0); quantile_depths / quantile_indices (num_rays, K) out, unfilled
 * entries -1 / 0xffffffff.  contribution (N) in the attribute dtype,
 * zero-initialised by the caller, or null.  distortion, W_total, S_total,
 * t_far (num_rays) f32 out.  path: null, or a record to write (vt_path). */
VT_API vt_status vt_trace_fwd(const vt_scene *scene, int attr_half, const void *diffuse,
                              const void *specular, int res, const float *rays, uint32_t num_rays,
                              const uint32_t *start, uint32_t num_quantiles,
                              const float *depth_quantiles, float weight_threshold,
                              uint32_t max_intersections, void *rgba, float *quantile_depths,
                              uint32_t *quantile_indices, uint32_t *num_intersections,
                              void *contribution, float *distortion, float *W_total,
                              float *S_total, float *t_far, const vt_debug *debug,
                              const vt_path *path, uint32_t *err, vt_stream stream);

/* Training backward.  Gradients are added to the outputs (zero-initialised
 * by the caller), or overwrite them with VT_BWD_OVERWRITE: points_grad (N,3) f32, diffuse/specular_grad in the attribute
 * dtype, density_grad (N) f32, point_error (N) attribute dtype or null
 * (accumulated only when ray_error is given).  path: null (walk every ray),
 * or the record written by the matching forward. */
VT_API vt_status vt_trace_bwd(const vt_scene *scene, int attr_half, const void *diffuse,
                              const void *specular, int res, const float *rays, uint32_t num_rays,
                              const uint32_t *start, uint32_t num_quantiles,
                              const float *depth_quantiles, const uint32_t *quantile_indices,
                              const void *rgba, const void *rgba_grad, const float *depth_grad,
                              const void *ray_error, float contribution_alpha_grad,
                              const float *distortion, const float *distortion_grad,
                              const float *W_total, const float *S_total, float weight_threshold,
                              uint32_t max_intersections, float *points_grad, void *diffuse_grad,
                              void *specular_grad, float *density_grad, void *point_error,
                              void *workspace, uint64_t workspace_bytes, const vt_path *path,
                              uint32_t flags, uint32_t *err, vt_stream stream);
/* vt_trace_bwd flags.  VT_BWD_OVERWRITE: the gradient outputs are
 * overwritten instead of accumulated into, so they need no zero
 * initialisation (requires the workspace). */
#define VT_BWD_OVERWRITE 1u
/* VT_BWD_KEEP_WORKSPACE (with VT_BWD_OVERWRITE): leave the texel and site
 * sums in the workspace instead of writing them to the outputs (density_grad
 * is still written); vt_grad_allreduce_peer then reduces them across ranks
 * straight into every rank's gradient bucket. */
#define VT_BWD_KEEP_WORKSPACE 2u
/* Optional scratch of vt_trace_bwd (256-byte aligned): with it the texel and
 * site gradients accumulate in padded fp32 rows with one vector atomic per
 * texel (instead of three scalar atomics) and are added to the outputs at the
 * end; fp16 gradients (point_error included) are then summed in fp32 and
 * rounded once.  Pass null
 * to accumulate straight into the outputs. */
VT_API uint64_t vt_trace_bwd_workspace_bytes(uint32_t num_points, int res);

/* ---- multi-GPU gradient reduction over peer memory ---- */

/* CUDA IPC of device buffers between the processes of one node: the handle
 * (64 bytes) and byte offset of `ptr` inside its allocation; a handle
 * opened by another process (vt_ipc_open, which maps the whole allocation;
 * add the offset) and its release.  No reference counterpart: the
 * reference trains on one GPU. */
VT_API vt_status vt_ipc_handle(const void *ptr, void *handle64, uint64_t *offset);
VT_API vt_status vt_ipc_open(const void *handle64, void **base);
VT_API vt_status vt_ipc_close(void *base);

#define VT_PEER_MAX 8
/* Every rank's backward workspace (written by vt_trace_bwd with
 * VT_BWD_KEEP_WORKSPACE), flat f32 gradient bucket [points 3N | density N |
 * diffuse 3R^2 N | specular 3R^2 N] and staging buffer (world slots of
 * vt_peer_staging_floats(num_points, res, world) floats), as device
 * addresses valid on the calling GPU (its own, or peers' opened with
 * vt_ipc_open).  Only the buckets and staging buffers are accessed across
 * GPUs.  fp32 attributes only. */
typedef struct {
    uint32_t world;
    uint32_t num_points;
    int32_t res;
    const void *workspace[VT_PEER_MAX];
    float *bucket[VT_PEER_MAX];
    float *staging[VT_PEER_MAX];
} vt_peer_grads;
/* Floats in one staging slot: the largest rank's share of the bucket. */
VT_API uint64_t vt_peer_staging_floats(uint32_t num_points, int res, uint32_t world);
/* The all-reduce of the training step, fused with the workspace compaction,
 * in two phases over peer memory.  Rank r owns a contiguous 1/world share of
 * the bucket.  Phase 0: rank r compacts its own workspace (and copies its
 * densities) and writes every other rank's share of it into slot r of that
 * rank's staging buffer (peer stores).  Phase 1: rank r sums its share over
 * the ranks in rank order 0..world-1 (its own workspace, the other ranks'
 * staging slots) and writes the sums into that share of every rank's bucket
 * (peer stores), so every rank ends with bit-identical buckets.  Ordering is
 * the caller's: every rank's phase 0 must be complete before any rank's
 * phase 1 (e.g. a stream-ordered collective as a fence), and every rank's
 * phase 1 before a bucket is read or a staging buffer written again.  The
 * kernels never wait on another GPU.  Replaces the vt_trace_bwd compaction
 * plus an NCCL all-reduce of the bucket. */
VT_API vt_status vt_grad_allreduce_peer(const vt_peer_grads *grads, uint32_t rank,
                                        uint32_t phase, vt_stream stream);

/* ---- cameras (ray generation for the benchmark views) ---- */

#define VT_CAMERA_PINHOLE 0   /* generate_camera_rays, vorotracing/utils/__init__.py:85-130 */
#define VT_CAMERA_FISHEYE 1   /* equidistant r = f * theta; no counterpart in the reference */
#define VT_CAMERA_ROLLING 2   /* pinhole, centre moving during the row readout; no counterpart */
#define VT_CAMERA_THIN_LENS 3 /* depth of field, spp lens samples per pixel; no counterpart */

typedef struct {
    float K[4];         /* fx, fy, cx, cy (pixels) */
    float c2w[12];      /* camera-to-world 3x4 row-major, OpenCV axes (x right, y down, z fwd) */
    uint32_t width, height, spp;
    int32_t model;      /* VT_CAMERA_* */
    float rs_duration;  /* rolling shutter: readout time of the whole frame (s) */
    float velocity[3];  /* rolling shutter: camera centre velocity (world units / s) */
    float lens_radius;  /* thin lens */
    float focus_distance;
    uint32_t seed;      /* thin lens sample jitter */
} vt_camera;

/* rays (height, width, spp, 6) f32: origin, unit direction. */
VT_API vt_status vt_raygen(const vt_camera *cam, float *rays, vt_stream stream);

/* Fused Adam step over flat fp32 buffers laid out in four groups ending at
 * group_ends[0..3] (= n), learning rates lrs[0..3], torch.optim.Adam's
 * update; then values of group clamp_group (or none, -1) are clamped to at
 * most clamp_max.  Replaces the reference's optimizer.step() + density
 * clamp (vorotracing/trainer.py:258-265, 503-527). */
VT_API vt_status vt_adam_step(float *params, const float *grads, float *exp_avg,
                              float *exp_avg_sq, uint64_t n, const uint64_t *group_ends,
                              const float *lrs, float beta1, float beta2, float eps,
                              uint32_t step, int clamp_group, float clamp_max, vt_stream stream);

/* ---- ray-origin cell lookup (nearest site) ---- */

/* Size of the BVH blob (internal nodes + leaf ids) for num_points sites. */
VT_API uint64_t vt_bvh_nodes_bytes(uint32_t num_points);
/* Scratch needed by vt_bvh_build. */
VT_API uint64_t vt_bvh_workspace_bytes(uint32_t num_points);
/* Build the BVH over points (N,3) f32 into `nodes` (256-byte aligned). */
VT_API vt_status vt_bvh_build(const float *points, uint32_t num_points, void *nodes,
                              uint64_t nodes_bytes, void *workspace, uint64_t workspace_bytes,
                              vt_stream stream);
/* Same build as vt_bvh_build, for callers that cannot allocate device
 * memory (an application that lends this library only its input and output
 * buffers, or a binding without a CUDA allocator): its scratch is a fixed
 * 40 MiB array inside the library, held on every GPU that loads it, so it
 * takes no workspace argument and accepts at most VT_BVH_NOALLOC_MAX_POINTS
 * sites (more: VT_ERR_INVALID).  The first call on a device looks up the
 * array's device address; make it before any stream capture.  Calls share
 * the array: calls that overlap on the GPU race, so serialise them.
 * No counterpart in the reference. */
#define VT_BVH_NOALLOC_MAX_POINTS 1048576u
VT_API vt_status vt_bvh_build_noalloc(const float *points, uint32_t num_points, void *nodes,
                                      uint64_t nodes_bytes, vt_stream stream);
/* out[q] = index of the site nearest to queries[q] (squared distance in
 * binary32, ties to the lowest index), int32. */
VT_API vt_status vt_bvh_query(const void *nodes, const float *points, uint32_t num_points,
                              const float *queries, uint32_t num_queries, int32_t *out,
                              uint32_t *err, vt_stream stream);
/* vt_bvh_query with a hint: hint (device, hint_count = 1 for all queries or
 * num_queries) names a site believed nearest, which bounds the search from
 * the start; the answer is the same.  Per-ray start cells of cameras whose
 * origins share a cell (rolling shutter, thin lens) cost a fraction of the
 * unhinted search.  No reference counterpart. */
VT_API vt_status vt_bvh_query_hint(const void *nodes, const float *points, uint32_t num_points,
                                   const float *queries, uint32_t num_queries,
                                   const uint32_t *hint, uint32_t hint_count, int32_t *out,
                                   uint32_t *err, vt_stream stream);

/* ---- Voronoi adjacency (replaces the external paragram package,
 *      vorotracing/cuda/__init__.py:16-46) ---- */

/* Scratch for vt_voronoi_adjacency / vt_voronoi_write (keep it between the two calls). */
VT_API uint64_t vt_voronoi_bytes(uint32_t num_points);
/* Voronoi face adjacency of the sites by per-cell clipping.  Writes the CSR
 * offsets (num_points + 1, device) and returns the entry count on the host
 * (*num_entries); neighbour ids of each row are ascending.  *unconverged
 * (host, optional) = cells left empty after every pass.  Synchronises the
 * stream (it reads sizes back to the host).  seed_adjacency / seed_offsets
 * (device CSR, optional, both or neither): initial guesses of each site's
 * neighbours (e.g. the adjacency before the sites moved, as paragram's
 * initial_guesses); they replace the nearest-site seeding and do not change
 * the result, which every cell's vertex verification fixes. */
VT_API vt_status vt_voronoi_adjacency(const float *points, uint32_t num_points,
                                      const uint32_t *seed_adjacency, const uint32_t *seed_offsets,
                                      void *workspace,
                                      uint64_t workspace_bytes, uint32_t *offsets,
                                      uint64_t *num_entries, uint32_t *unconverged,
                                      vt_stream stream);
/* Write the neighbour ids into adjacency (>= *num_entries entries). */
VT_API vt_status vt_voronoi_write(const void *workspace, uint32_t num_points,
                                  const uint32_t *offsets, uint32_t *adjacency, vt_stream stream);

/* ---- layout transforms ---- */

/* Column-wise min and max of a (rows, cols<=4) f32 matrix -> out[2*c], out[2*c+1].
 * workspace: 256 bytes. */
VT_API vt_status vt_minmax_f32(const float *x, uint64_t rows, int cols, void *workspace,
                               float *out, vt_stream stream);
/* Scratch for vt_morton_codes / vt_morton_perm / vt_permute_csr. */
VT_API uint64_t vt_morton_workspace_bytes(uint32_t num_points);
/* 30-bit Morton codes (int64) of the bbox-normalised sites. */
VT_API vt_status vt_morton_codes(const float *points, uint32_t num_points, int64_t *codes,
                                 void *workspace, vt_stream stream);
/* perm = stable argsort(codes), inv_perm[perm[i]] = i (u32). */
VT_API vt_status vt_morton_perm(const int64_t *codes, uint32_t num_points, uint32_t *perm,
                                uint32_t *inv_perm, void *workspace, uint64_t workspace_bytes,
                                vt_stream stream);
/* dst row i = src row perm[i], rows of row_bytes bytes. */
VT_API vt_status vt_gather_rows(const void *src, void *dst, const uint32_t *perm, uint32_t num_rows,
                                uint32_t row_bytes, vt_stream stream);
/* CSR of the permuted scene: new row i = old row perm[i], ids mapped by inv_perm. */
VT_API vt_status vt_permute_csr(const uint32_t *offsets, const uint32_t *adjacency,
                                uint32_t num_points, const uint32_t *perm, const uint32_t *inv_perm,
                                uint32_t *new_offsets, uint32_t *new_adjacency, void *workspace,
                                uint64_t workspace_bytes, vt_stream stream);
/* Thread-to-pixel order of tile_h x tile_w warp tiles over a height x width image. */
VT_API vt_status vt_tile_perm(uint32_t height, uint32_t width, uint32_t tile_h, uint32_t tile_w,
                              uint32_t *perm, vt_stream stream);
/* f32 rgb texels -> binary16 Half4Texel rows (rgb + zero pad). */
VT_API vt_status vt_pad_f16x4(const float *src, uint64_t texels, void *dst, vt_stream stream);
/* q8 maps (N, 3*R*R) u8 -> (N, 4*R*R) u8, a zero 4th byte per texel (the
 * layout of vt_trace_infer_q8x4); texels = N*R*R, dst 4-byte aligned. */
VT_API vt_status vt_pad_u8x4(const uint8_t *src, uint64_t texels, void *dst, vt_stream stream);
/* dst = clamp(rint((src - offset) / scale), 0, 255). */
VT_API vt_status vt_quantize_u8(const float *src, uint64_t count, float scale, float offset,
                                uint8_t *dst, vt_stream stream);

#ifdef __cplusplus
}
#endif

#endif
