// vt_infer.cu -- fp16 and q8 inference kernels and their C entry points
// (reference kernels: tracing_octmap.cu:552-610 and :723-779; host
// wrappers :642-717 and :781-854).
//
// One thread per ray; with a ray permutation thread t traces ray perm[t]
// (tracing_octmap.cu:574), so a warp covers a compact 4x8 pixel tile while
// inputs and outputs stay in image order.  The q8 path takes the same
// optional permutation (the reference's has none; outputs are identical
// because rays are independent).
#include "vt_abi.cuh"
#include "vt_integrators.cuh"
#include "vt_walk.cuh"

namespace vt {

constexpr int kInferBlock = 128;

struct InferArgs {
    const float *points;
    const float *density;
    const uint32_t *offs;
    const uint4 *faces;
    uint32_t n_points;
    const float *rays;
    uint32_t num_rays;
    const uint32_t *start;
    const uint32_t *perm;
    float wt, skip;
    uint32_t max_steps;
    uint2 *rgba;  // 4 x binary16 per ray
    WalkDebug dbg;
    uint32_t *n_out;
    uint32_t *err;
};

template <int R, class Tex, bool kDebug>
__global__ void __launch_bounds__(kInferBlock) infer_kernel(InferArgs a, Tex tex)
{
    uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= a.num_rays) return;
    uint32_t ray_id = a.perm ? __ldg(a.perm + tid) : tid;
    if (ray_id >= a.num_rays) {
        report(a.err, VT_ERR_DATA);
        return;
    }
    Ray ray = load_ray(a.rays, ray_id);
    uint32_t start = __ldg(a.start + ray_id);
    if (start >= a.n_points) {
        report(a.err, VT_ERR_DATA);
        a.rgba[ray_id] = make_uint2(0, 0);
        return;
    }
    InferInteg<R, Tex> I(ray, tex, a.wt, a.skip);
    uint32_t n = walk<InferInteg<R, Tex>, kDebug>(ray, a.faces, a.offs, a.points, a.density, start,
                                                  a.max_steps, I, ray_id, a.dbg);
    uint2 o;
    o.x = (uint32_t)f2h(I.acc.x) | ((uint32_t)f2h(I.acc.y) << 16);
    o.y = (uint32_t)f2h(I.acc.z) | ((uint32_t)f2h(1.0f - I.T) << 16);
    a.rgba[ray_id] = o;
    if (kDebug && a.n_out) a.n_out[ray_id] = n;
}

template <int R, class Tex>
vt_status launch_infer(const InferArgs &a, const Tex &tex, bool debug, cudaStream_t stream)
{
    unsigned grid = grid_for(a.num_rays, kInferBlock);
    if (debug)
        infer_kernel<R, Tex, true><<<grid, kInferBlock, 0, stream>>>(a, tex);
    else
        infer_kernel<R, Tex, false><<<grid, kInferBlock, 0, stream>>>(a, tex);
    return check_launch("infer_kernel");
}

vt_status fill_args(InferArgs &a, const vt_scene *scene, const float *rays, uint32_t num_rays,
                    const uint32_t *start, const uint32_t *perm, float wt, uint32_t max_int,
                    float skip, void *rgba, const vt_debug *dbg, uint32_t *err, const char *who)
{
    VT_REQUIRE(scene && scene->points && scene->density && scene->offsets && scene->faces,
               "%s: incomplete scene", who);
    VT_REQUIRE(scene->num_points > 0, "%s: empty scene", who);
    VT_REQUIRE(((uintptr_t)scene->faces & 15u) == 0, "%s: faces must be 16-byte aligned", who);
    VT_REQUIRE(num_rays == 0 || (rays && start && rgba), "%s: null ray buffers", who);
    VT_REQUIRE(((uintptr_t)rays & 7u) == 0, "%s: rays must be 8-byte aligned", who);
    VT_REQUIRE(((uintptr_t)rgba & 7u) == 0, "%s: rgba must be 8-byte aligned", who);
    a.points = scene->points;
    a.density = scene->density;
    a.offs = scene->offsets;
    a.faces = (const uint4 *)scene->faces;
    a.n_points = scene->num_points;
    a.rays = rays;
    a.num_rays = num_rays;
    a.start = start;
    a.perm = perm;
    a.wt = wt;
    a.skip = skip;
    a.max_steps = max_int;
    a.rgba = (uint2 *)rgba;
    a.dbg = WalkDebug{nullptr, 0, nullptr, nullptr, nullptr, nullptr};
    a.n_out = nullptr;
    if (dbg) {
        a.dbg = WalkDebug{dbg->seq, dbg->seq_cap, dbg->seq_len, (uint4 *)dbg->stats,
                          dbg->visited, dbg->textured};
        a.n_out = dbg->num_intersections;
        VT_REQUIRE(((uintptr_t)dbg->stats & 15u) == 0, "%s: stats must be 16-byte aligned", who);
    }
    a.err = err;
    return VT_OK;
}

}  // namespace vt

extern "C" vt_status vt_trace_infer_f16(const vt_scene *scene, const void *diffuse,
                                        const void *specular, int res, const float *rays,
                                        uint32_t num_rays, const uint32_t *start,
                                        const uint32_t *ray_perm, float weight_threshold,
                                        uint32_t max_intersections, float cell_skip_threshold,
                                        void *rgba, const vt_debug *debug, uint32_t *err,
                                        vt_stream stream)
{
    vt::InferArgs a;
    vt_status st = vt::fill_args(a, scene, rays, num_rays, start, ray_perm, weight_threshold,
                                 max_intersections, cell_skip_threshold, rgba, debug, err,
                                 "vt_trace_infer_f16");
    if (st != VT_OK) return st;
    VT_REQUIRE(diffuse && specular, "vt_trace_infer_f16: null textures");
    VT_REQUIRE((((uintptr_t)diffuse | (uintptr_t)specular) & 7u) == 0,
               "vt_trace_infer_f16: textures must be 8-byte aligned");
    if (num_rays == 0) return VT_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (res == 8) {
        vt::TexF16x4<8> t{(const uint2 *)diffuse, (const uint2 *)specular};
        return vt::launch_infer<8>(a, t, debug != nullptr, s);
    }
    if (res == 4) {
        vt::TexF16x4<4> t{(const uint2 *)diffuse, (const uint2 *)specular};
        return vt::launch_infer<4>(a, t, debug != nullptr, s);
    }
    return vt::set_error(VT_ERR_INVALID, "vt_trace_infer_f16: res must be 4 or 8, got %d", res);
}

extern "C" vt_status vt_trace_infer_q8(const vt_scene *scene, const uint8_t *diffuse,
                                       const uint8_t *specular, int res, float diff_scale,
                                       float diff_offset, float spec_scale, float spec_offset,
                                       const float *rays, uint32_t num_rays, const uint32_t *start,
                                       const uint32_t *ray_perm, float weight_threshold,
                                       uint32_t max_intersections, float cell_skip_threshold,
                                       void *rgba, const vt_debug *debug, uint32_t *err,
                                       vt_stream stream)
{
    vt::InferArgs a;
    vt_status st = vt::fill_args(a, scene, rays, num_rays, start, ray_perm, weight_threshold,
                                 max_intersections, cell_skip_threshold, rgba, debug, err,
                                 "vt_trace_infer_q8");
    if (st != VT_OK) return st;
    VT_REQUIRE(diffuse && specular, "vt_trace_infer_q8: null textures");
    if (num_rays == 0) return VT_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (res == 8) {
        vt::TexQ8<8> t{diffuse, specular, diff_scale, diff_offset, spec_scale, spec_offset};
        return vt::launch_infer<8>(a, t, debug != nullptr, s);
    }
    if (res == 4) {
        vt::TexQ8<4> t{diffuse, specular, diff_scale, diff_offset, spec_scale, spec_offset};
        return vt::launch_infer<4>(a, t, debug != nullptr, s);
    }
    return vt::set_error(VT_ERR_INVALID, "vt_trace_infer_q8: res must be 4 or 8, got %d", res);
}

extern "C" vt_status vt_trace_infer_q8x4(const vt_scene *scene, const void *diffuse,
                                         const void *specular, int res, float diff_scale,
                                         float diff_offset, float spec_scale, float spec_offset,
                                         const float *rays, uint32_t num_rays,
                                         const uint32_t *start, const uint32_t *ray_perm,
                                         float weight_threshold, uint32_t max_intersections,
                                         float cell_skip_threshold, void *rgba,
                                         const vt_debug *debug, uint32_t *err, vt_stream stream)
{
    vt::InferArgs a;
    vt_status st = vt::fill_args(a, scene, rays, num_rays, start, ray_perm, weight_threshold,
                                 max_intersections, cell_skip_threshold, rgba, debug, err,
                                 "vt_trace_infer_q8x4");
    if (st != VT_OK) return st;
    VT_REQUIRE(diffuse && specular, "vt_trace_infer_q8x4: null textures");
    VT_REQUIRE((((uintptr_t)diffuse | (uintptr_t)specular) & 3u) == 0,
               "vt_trace_infer_q8x4: textures must be 4-byte aligned");
    if (num_rays == 0) return VT_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (res == 8) {
        vt::TexQ8x4<8> t{(const uint32_t *)diffuse, (const uint32_t *)specular, diff_scale,
                         diff_offset, spec_scale, spec_offset};
        return vt::launch_infer<8>(a, t, debug != nullptr, s);
    }
    if (res == 4) {
        vt::TexQ8x4<4> t{(const uint32_t *)diffuse, (const uint32_t *)specular, diff_scale,
                         diff_offset, spec_scale, spec_offset};
        return vt::launch_infer<4>(a, t, debug != nullptr, s);
    }
    return vt::set_error(VT_ERR_INVALID, "vt_trace_infer_q8x4: res must be 4 or 8, got %d", res);
}

// ---------------------------------------------------------------- depth
namespace vt {

__global__ void __launch_bounds__(kInferBlock)
    depth_kernel(InferArgs a, const float *__restrict__ thr, uint32_t K, int mode, float *out)
{
    uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= a.num_rays) return;
    uint32_t ray_id = a.perm ? __ldg(a.perm + tid) : tid;
    if (ray_id >= a.num_rays) {
        report(a.err, VT_ERR_DATA);
        return;
    }
    Ray ray = load_ray(a.rays, ray_id);
    uint32_t start = __ldg(a.start + ray_id);
    if (start >= a.n_points) {
        report(a.err, VT_ERR_DATA);
        out[ray_id] = -1.0f;
        return;
    }
    DepthInteg I(thr, K, a.wt);
    walk<DepthInteg, false>(ray, a.faces, a.offs, a.points, a.density, start, a.max_steps, I,
                            ray_id, a.dbg);
    float v;
    if (mode == VT_DEPTH_FIRST_QUANTILE)
        v = I.qi > 0 ? I.first : -1.0f;
    else
        v = I.cnt ? I.sum / (float)I.cnt : -1.0f;
    out[ray_id] = v;
}

}  // namespace vt

extern "C" vt_status vt_trace_depth(const vt_scene *scene, const float *rays, uint32_t num_rays,
                                    const uint32_t *start, const uint32_t *ray_perm,
                                    const float *thresholds, uint32_t num_thresholds, int mode,
                                    float weight_threshold, uint32_t max_intersections,
                                    float *depth, uint32_t *err, vt_stream stream)
{
    vt::InferArgs a;
    vt_status st = vt::fill_args(a, scene, rays, num_rays, start, ray_perm, weight_threshold,
                                 max_intersections, 0.0f, depth, nullptr, err, "vt_trace_depth");
    if (st != VT_OK) return st;
    VT_REQUIRE(thresholds && num_thresholds > 0, "vt_trace_depth: thresholds required");
    VT_REQUIRE(mode == VT_DEPTH_FIRST_QUANTILE || mode == VT_DEPTH_MEAN,
               "vt_trace_depth: unknown mode %d", mode);
    if (num_rays == 0) return VT_OK;
    vt::depth_kernel<<<vt::grid_for(num_rays, vt::kInferBlock), vt::kInferBlock, 0,
                       (cudaStream_t)stream>>>(a, thresholds, num_thresholds, mode, depth);
    return vt::check_launch("depth_kernel");
}
