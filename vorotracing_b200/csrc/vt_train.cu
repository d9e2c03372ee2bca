// vt_train.cu -- training forward / backward kernels and C entry points
// (reference kernels tracing_octmap.cu:151-230 and :232-340, host wrappers
// :355-546 and :860-1103).  One thread per ray, rays in input order.  The
// packed face rows replace the reference's per-call adj_diff prefetch; the
// host layer rebuilds them from the current sites before each call, as the
// reference re-runs its prefetch kernel on every fwd / bwd call.
#include "vt_abi.cuh"
#include "vt_train_integ.cuh"
#include "vt_walk.cuh"

namespace vt {

constexpr int kTrainBlock = 128;
#ifndef VT_BWD_MIN_BLOCKS
#define VT_BWD_MIN_BLOCKS 4  // C4 replay backward: 4 blocks 15.38 ms, 5 blocks 16.27 ms, 6 blocks 16.55 ms (same box)
#endif
#ifndef VT_FWD_MIN_BLOCKS
#define VT_FWD_MIN_BLOCKS 8  // measured: 6.98 -> 6.41 ms on the C2 scene (fp32, tile order)
#endif

struct TrainCommon {
    const float *points;
    const float *density;
    const uint32_t *offs;
    const uint4 *faces;
    uint32_t n_points;
    const float *rays;
    uint32_t num_rays;
    const uint32_t *start;
    uint32_t K;
    const float *dq;
    float wt;
    uint32_t max_steps;
    uint32_t *err;
};

template <class AT> struct FwdOut {
    AT *rgba;
    float *qdepth;
    uint32_t *qidx;
    uint32_t *n_int;
    AT *contrib;
    float *dist, *W, *S, *tfar;
    WalkDebug dbg;
    PathRec rec;
};

#ifndef VT_FWD_REC_MIN_BLOCKS
#define VT_FWD_REC_MIN_BLOCKS 7  // the record store needs a few more registers
#endif

template <class AT, int R, bool kDebug, bool kRec>
__global__ void __launch_bounds__(kTrainBlock, kRec ? VT_FWD_REC_MIN_BLOCKS : VT_FWD_MIN_BLOCKS)
    fwd_kernel(TrainCommon a, TexPlain<AT, R> tex, FwdOut<AT> o)
{
    uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.num_rays) return;
    Ray ray = load_ray(a.rays, r);
    uint32_t start = __ldg(a.start + r);
    const float *qthr = a.dq ? a.dq + (size_t)r * a.K : nullptr;
    float *qd = o.qdepth ? o.qdepth + (size_t)r * a.K : nullptr;
    uint32_t *qi = o.qidx ? o.qidx + (size_t)r * a.K : nullptr;
    FwdInteg<AT, R> I(ray, tex, a.wt, qthr, a.dq ? a.K : 0, qd, qi, o.contrib);
    uint32_t n = 0;
    if (start >= a.n_points) {
        report(a.err, VT_ERR_DATA);
        if (kRec) o.rec.len[r] = kPathWalk;
    } else {
        n = walk<FwdInteg<AT, R>, kDebug, kRec>(ray, a.faces, a.offs, a.points, a.density, start,
                                                a.max_steps, I, r, o.dbg, o.rec);
    }
    if (kRec && (o.rec.len[r] > o.rec.cap || I.T == a.wt)) o.rec.len[r] |= kPathWalk;
    for (uint32_t i = I.qi; i < a.K; ++i) {
        qd[i] = -1.0f;
        qi[i] = 0xffffffffu;
    }
    AT *out = o.rgba + (size_t)r * 4;
    out[0] = fromf<AT>(I.acc.x);
    out[1] = fromf<AT>(I.acc.y);
    out[2] = fromf<AT>(I.acc.z);
    out[3] = fromf<AT>(1.0f - I.T);
    if (o.n_int) o.n_int[r] = n;
    o.dist[r] = 2.0f * I.dist + I.self / 3.0f;
    o.W[r] = I.W;
    o.S[r] = I.S;
    o.tfar[r] = I.tfar;
}

template <class AT> struct BwdIn {
    const uint32_t *qidx;
    const AT *rgba;
    const AT *rgba_grad;
    const float *depth_grad;
    const AT *ray_error;
    float contribution_alpha_grad;
    const float *dist, *dist_grad, *W, *S;
    float *points_grad;
    AT *diffuse_grad, *specular_grad;
    float *density_grad;
    AT *point_error;
    float4 *sdiff, *sspec, *spts;  // padded scratch or null
    float *sperr;                  // fp32 point_error scratch or null
    PathRec rec;                   // forward's path record or null cells
};

// Backward launch modes: walk every ray; replay the rays of a path record;
// walk only the rays the record flags.
constexpr int kBwdWalkAll = 0, kBwdReplay = 1, kBwdWalkFlagged = 2;

template <class AT, int R, int F, int M>
__global__ void __launch_bounds__(kTrainBlock, VT_BWD_MIN_BLOCKS)
    bwd_kernel(TrainCommon a, TexPlain<AT, R> tex, BwdIn<AT> b)
{
    __shared__ typename BwdInteg<AT, R, F>::AggLane agg[kTrainBlock];
    uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.num_rays) return;
    uint32_t L = 0;
    if (M != kBwdWalkAll) {
        L = __ldg(b.rec.len + r);
        if ((M == kBwdReplay) == ((L & kPathWalk) != 0)) return;
    }
    Ray ray = load_ray(a.rays, r);
    uint32_t start = __ldg(a.start + r);
    if (start >= a.n_points) {
        report(a.err, VT_ERR_DATA);
        return;
    }
    BwdInteg<AT, R, F> I;
    I.ray = ray;
    I.tex = tex;
    I.wt = a.wt;
    I.acc = mk(0.f, 0.f, 0.f);
    I.T = 1.0f;
    I.ntex = 0;
    float c[4], g[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        c[k] = tof<AT>(b.rgba[(size_t)r * 4 + k]);
        g[k] = tof<AT>(b.rgba_grad[(size_t)r * 4 + k]);
    }
    g[3] += b.contribution_alpha_grad;
    I.fwd_rgb = mk(c[0], c[1], c[2]);
    I.fwd_a = c[3];
    I.g_rgb = mk(g[0], g[1], g[2]);
    I.g_a = g[3];
    I.ray_error = b.ray_error ? tof<AT>(b.ray_error[r]) : 0.0f;
    float cdg = 0.0f;
    for (uint32_t i = 0; (F & kBwdDepth) != 0 && i < a.K; ++i) {
        uint32_t pi = b.qidx[(size_t)r * a.K + i];
        if (pi != 0xffffffffu) cdg += b.depth_grad[(size_t)r * a.K + i] / __ldg(a.density + pi);
    }
    I.cur_dg = cdg;
    I.K = a.dq ? a.K : 0;
    I.qthr = a.dq ? a.dq + (size_t)r * a.K : nullptr;
    I.dgrad = b.depth_grad ? b.depth_grad + (size_t)r * a.K : nullptr;
    I.qi = 0;
    I.qv = I.K > 0 ? I.qthr[0] : 0.0f;
    I.W = 0.f;
    I.S = 0.f;
    I.Wt = b.W ? b.W[r] : 0.0f;
    I.St = b.S ? b.S[r] : 0.0f;
    float fd = b.dist ? b.dist[r] : 0.0f;
    I.dgr = b.dist_grad ? b.dist_grad[r] : 0.0f;
    I.Dt = (2.0f * fd) * I.dgr;
    I.Drun = 0.0f;
    I.s_prev = 0.0f;
    I.pgrad = b.points_grad;
    I.ddiff = b.diffuse_grad;
    I.dspec = b.specular_grad;
    I.dden = b.density_grad;
    I.perr = b.point_error;
    I.sdiff = b.sdiff;
    I.sspec = b.sspec;
    I.spts = b.spts;
    I.sperr = b.sperr;
    I.agg = agg + (threadIdx.x & ~31u);
    I.prev_geom = I.prev_grad = I.cur_grad = I.next_grad = mk(0.f, 0.f, 0.f);
    I.prev_idx = 0xffffffffu;
    float tu, tv;
    oct_encode<R>(mk(-ray.d.x, -ray.d.y, -ray.d.z), tu, tv);
    I.spec = make_bilin<R>(tu, tv);
    if (M == kBwdReplay) {
        WalkState w;
        walk_replay<BwdInteg<AT, R, F>>(ray, a.points, a.density, start, min(L, a.max_steps), I,
                                        b.rec.steps + r, b.rec.stride, w);
    } else if (M == kBwdWalkFlagged) {
        // replay what the record holds, then walk on with the face scan
        WalkState w;
        const uint32_t Lr = min(min(L & ~kPathWalk, b.rec.cap), a.max_steps);
        if (walk_replay<BwdInteg<AT, R, F>>(ray, a.points, a.density, start, Lr, I,
                                            b.rec.steps + r, b.rec.stride, w)) {
            w.begin = __ldg(a.offs + w.cur);
            w.deg = __ldg(a.offs + w.cur + 1) - w.begin;
            WalkDebug none{nullptr, 0, nullptr, nullptr, nullptr, nullptr};
            walk_from<BwdInteg<AT, R, F>, false, false>(w, ray, a.faces, a.points, a.density,
                                                         a.max_steps, I, r, none,
                                                         PathRec{nullptr, 0, 0, nullptr});
        }
    } else {
        WalkDebug none{nullptr, 0, nullptr, nullptr, nullptr, nullptr};
        walk<BwdInteg<AT, R, F>, false>(ray, a.faces, a.offs, a.points, a.density, start,
                                        a.max_steps, I, r, none);
    }
}

// out[t*3 + c] += scratch[t].c for every texel (or site) t; kSet: = instead.
template <class AT, bool kSet>
__global__ void compact4_kernel(const float4 *__restrict__ scratch, uint64_t n, AT *__restrict__ out)
{
    uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    float4 v = scratch[t];
    AT *o = out + t * 3;
    if (kSet) {
        o[0] = fromf<AT>(v.x);
        o[1] = fromf<AT>(v.y);
        o[2] = fromf<AT>(v.z);
    } else {
        o[0] = fromf<AT>(tof<AT>(o[0]) + v.x);
        o[1] = fromf<AT>(tof<AT>(o[1]) + v.y);
        o[2] = fromf<AT>(tof<AT>(o[2]) + v.z);
    }
}

// out[t] (+)= scratch[t]: the fp32 point_error sums rounded once.
template <class AT, bool kSet>
__global__ void compact1_kernel(const float *__restrict__ scratch, uint64_t n, AT *__restrict__ out)
{
    uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    out[t] = kSet ? fromf<AT>(scratch[t]) : fromf<AT>(tof<AT>(out[t]) + scratch[t]);
}

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

vt_status fill_common(TrainCommon &a, const vt_scene *scene, const float *rays, uint32_t nr,
                      const uint32_t *start, uint32_t K, const float *dq, float wt,
                      uint32_t max_int, uint32_t *err, const char *who)
{
    VT_REQUIRE(scene && scene->points && scene->density && scene->offsets && scene->faces,
               "%s: incomplete scene", who);
    VT_REQUIRE(scene->num_points > 0, "%s: empty scene", who);
    VT_REQUIRE(((uintptr_t)scene->faces & 15u) == 0, "%s: faces must be 16-byte aligned", who);
    VT_REQUIRE(nr == 0 || (rays && start), "%s: null ray buffers", who);
    VT_REQUIRE(((uintptr_t)rays & 7u) == 0, "%s: rays must be 8-byte aligned", who);
    VT_REQUIRE(K == 0 || dq, "%s: depth quantiles missing", who);
    a = TrainCommon{scene->points, scene->density, scene->offsets, (const uint4 *)scene->faces,
                    scene->num_points, rays, nr, start, K, dq, wt, max_int, err};
    return VT_OK;
}

template <class AT, int R>
vt_status launch_fwd(const TrainCommon &a, const void *dif, const void *spe, const FwdOut<AT> &o,
                     bool debug, cudaStream_t s)
{
    TexPlain<AT, R> t{(const AT *)dif, (const AT *)spe};
    unsigned g = grid_for(a.num_rays, kTrainBlock);
    if (debug)
        o.rec.steps ? fwd_kernel<AT, R, true, true><<<g, kTrainBlock, 0, s>>>(a, t, o)
                    : fwd_kernel<AT, R, true, false><<<g, kTrainBlock, 0, s>>>(a, t, o);
    else
        o.rec.steps ? fwd_kernel<AT, R, false, true><<<g, kTrainBlock, 0, s>>>(a, t, o)
                    : fwd_kernel<AT, R, false, false><<<g, kTrainBlock, 0, s>>>(a, t, o);
    return check_launch("fwd_kernel");
}

template <class AT, int R>
vt_status launch_bwd(const TrainCommon &a, const void *dif, const void *spe, BwdIn<AT> b,
                     void *ws, bool overwrite, bool keep_ws, cudaStream_t s)
{
    TexPlain<AT, R> t{(const AT *)dif, (const AT *)spe};
    const uint64_t ntex = (uint64_t)a.n_points * R * R;
    if (ws) {
        char *w = (char *)ws;
        b.sdiff = (float4 *)w;
        b.sspec = (float4 *)(w + a256(ntex * 16));
        b.spts = (float4 *)(w + 2 * a256(ntex * 16));
        const size_t perr_off = 2 * a256(ntex * 16) + a256((size_t)a.n_points * 16);
        b.sperr = b.point_error ? (float *)(w + perr_off) : nullptr;
        cudaError_t e = cudaMemsetAsync(
            ws, 0, perr_off + (b.point_error ? a256((size_t)a.n_points * 4) : 0), s);
        if (e == cudaSuccess && overwrite)  // the outputs the kernels add to directly
            e = cudaMemsetAsync(b.density_grad, 0, (size_t)a.n_points * 4, s);
        if (e != cudaSuccess) return set_error(VT_ERR_CUDA, "vt_trace_bwd memset: %s", cudaGetErrorString(e));
    } else {
        b.sdiff = b.sspec = b.spts = nullptr;
        b.sperr = nullptr;
    }
    const int F = (a.K > 0 && a.dq ? kBwdDepth : 0) | (b.dist_grad ? kBwdDist : 0) |
                  (b.ray_error && b.point_error ? kBwdErr : 0);
    const unsigned g = grid_for(a.num_rays, kTrainBlock);
    switch (F) {
#define VT_BWD_CASE(f)                                                                             \
    case f:                                                                                        \
        if (b.rec.steps) {                                                                         \
            bwd_kernel<AT, R, f, kBwdReplay><<<g, kTrainBlock, 0, s>>>(a, t, b);                   \
            bwd_kernel<AT, R, f, kBwdWalkFlagged><<<g, kTrainBlock, 0, s>>>(a, t, b);              \
        } else {                                                                                   \
            bwd_kernel<AT, R, f, kBwdWalkAll><<<g, kTrainBlock, 0, s>>>(a, t, b);                  \
        }                                                                                          \
        break;
        VT_BWD_CASE(0) VT_BWD_CASE(1) VT_BWD_CASE(2) VT_BWD_CASE(3)
        VT_BWD_CASE(4) VT_BWD_CASE(5) VT_BWD_CASE(6) VT_BWD_CASE(7)
#undef VT_BWD_CASE
    }
    if (keep_ws) {
        // the texel, site and point_error sums stay in the workspace for
        // vt_grad_allreduce_peer, which reduces and compacts them across ranks
    } else if (ws && overwrite) {
        compact4_kernel<AT, true><<<grid_for(ntex, 256), 256, 0, s>>>(b.sdiff, ntex, b.diffuse_grad);
        compact4_kernel<AT, true><<<grid_for(ntex, 256), 256, 0, s>>>(b.sspec, ntex, b.specular_grad);
        compact4_kernel<float, true><<<grid_for(a.n_points, 256), 256, 0, s>>>(b.spts, a.n_points,
                                                                                b.points_grad);
        if (b.sperr)
            compact1_kernel<AT, true><<<grid_for(a.n_points, 256), 256, 0, s>>>(
                b.sperr, a.n_points, b.point_error);
    } else if (ws) {
        compact4_kernel<AT, false><<<grid_for(ntex, 256), 256, 0, s>>>(b.sdiff, ntex, b.diffuse_grad);
        compact4_kernel<AT, false><<<grid_for(ntex, 256), 256, 0, s>>>(b.sspec, ntex, b.specular_grad);
        compact4_kernel<float, false><<<grid_for(a.n_points, 256), 256, 0, s>>>(b.spts, a.n_points,
                                                                                 b.points_grad);
        if (b.sperr)
            compact1_kernel<AT, false><<<grid_for(a.n_points, 256), 256, 0, s>>>(
                b.sperr, a.n_points, b.point_error);
    }
    return check_launch("bwd_kernel");
}

}  // namespace vt

extern "C" vt_status vt_trace_fwd(const vt_scene *scene, int attr_half, const void *diffuse,
                                  const void *specular, int res, const float *rays,
                                  uint32_t num_rays, const uint32_t *start,
                                  uint32_t num_quantiles, const float *depth_quantiles,
                                  float weight_threshold, uint32_t max_intersections, void *rgba,
                                  float *quantile_depths, uint32_t *quantile_indices,
                                  uint32_t *num_intersections, void *contribution,
                                  float *distortion, float *W_total, float *S_total, float *t_far,
                                  const vt_debug *debug, const vt_path *path, uint32_t *err,
                                  vt_stream stream)
{
    vt::TrainCommon a;
    vt_status st = vt::fill_common(a, scene, rays, num_rays, start, num_quantiles, depth_quantiles,
                                   weight_threshold, max_intersections, err, "vt_trace_fwd");
    if (st != VT_OK) return st;
    VT_REQUIRE(diffuse && specular, "vt_trace_fwd: null textures");
    VT_REQUIRE(num_rays == 0 || (rgba && distortion && W_total && S_total && t_far),
               "vt_trace_fwd: null outputs");
    VT_REQUIRE(num_quantiles == 0 || (quantile_depths && quantile_indices),
               "vt_trace_fwd: null depth outputs");
    if (num_rays == 0) return VT_OK;
    vt::WalkDebug dbg{nullptr, 0, nullptr, nullptr, nullptr, nullptr};
    if (debug)
        dbg = vt::WalkDebug{debug->seq, debug->seq_cap, debug->seq_len, (uint4 *)debug->stats,
                            debug->visited, debug->textured};
    vt::PathRec rec{nullptr, 0, 0, nullptr};
    if (path && path->steps && path->cap) {
        VT_REQUIRE(path->len, "vt_trace_fwd: path record without len");
        VT_REQUIRE(((uintptr_t)path->steps & 15u) == 0, "vt_trace_fwd: path steps must be 16-byte aligned");
        rec = vt::PathRec{(uint4 *)path->steps, path->cap, num_rays, path->len};
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (attr_half) {
        vt::FwdOut<__half> o{(__half *)rgba, quantile_depths, quantile_indices, num_intersections,
                             (__half *)contribution, distortion, W_total, S_total, t_far, dbg, rec};
        if (res == 8) return vt::launch_fwd<__half, 8>(a, diffuse, specular, o, debug, s);
        if (res == 4) return vt::launch_fwd<__half, 4>(a, diffuse, specular, o, debug, s);
    } else {
        vt::FwdOut<float> o{(float *)rgba, quantile_depths, quantile_indices, num_intersections,
                            (float *)contribution, distortion, W_total, S_total, t_far, dbg, rec};
        if (res == 8) return vt::launch_fwd<float, 8>(a, diffuse, specular, o, debug, s);
        if (res == 4) return vt::launch_fwd<float, 4>(a, diffuse, specular, o, debug, s);
    }
    return vt::set_error(VT_ERR_INVALID, "vt_trace_fwd: res must be 4 or 8, got %d", res);
}

extern "C" uint64_t vt_trace_bwd_workspace_bytes(uint32_t num_points, int res)
{
    const uint64_t ntex = (uint64_t)num_points * res * res;
    return 2 * vt::a256(ntex * 16) + vt::a256((size_t)num_points * 16) +
           vt::a256((size_t)num_points * 4);
}

extern "C" vt_status vt_trace_bwd(const vt_scene *scene, int attr_half, const void *diffuse,
                                  const void *specular, int res, const float *rays,
                                  uint32_t num_rays, const uint32_t *start,
                                  uint32_t num_quantiles, const float *depth_quantiles,
                                  const uint32_t *quantile_indices, const void *rgba,
                                  const void *rgba_grad, const float *depth_grad,
                                  const void *ray_error, float contribution_alpha_grad,
                                  const float *distortion, const float *distortion_grad,
                                  const float *W_total, const float *S_total,
                                  float weight_threshold, uint32_t max_intersections,
                                  float *points_grad, void *diffuse_grad, void *specular_grad,
                                  float *density_grad, void *point_error, void *workspace,
                                  uint64_t workspace_bytes, const vt_path *path, uint32_t flags,
                                  uint32_t *err, vt_stream stream)
{
    vt::TrainCommon a;
    vt_status st = vt::fill_common(a, scene, rays, num_rays, start, num_quantiles, depth_quantiles,
                                   weight_threshold, max_intersections, err, "vt_trace_bwd");
    if (st != VT_OK) return st;
    VT_REQUIRE(res == 4 || res == 8, "vt_trace_bwd: res must be 4 or 8, got %d", res);
    VT_REQUIRE(!workspace || (((uintptr_t)workspace & 255u) == 0 &&
                              workspace_bytes >= vt_trace_bwd_workspace_bytes(scene->num_points, res)),
               "vt_trace_bwd: workspace must be 256-byte aligned and vt_trace_bwd_workspace_bytes large");
    VT_REQUIRE(!(flags & VT_BWD_OVERWRITE) || workspace,
               "vt_trace_bwd: VT_BWD_OVERWRITE needs the workspace");
    const bool overwrite = (flags & VT_BWD_OVERWRITE) != 0;
    const bool keep_ws = (flags & VT_BWD_KEEP_WORKSPACE) != 0;
    VT_REQUIRE(!keep_ws || (overwrite && workspace),
               "vt_trace_bwd: VT_BWD_KEEP_WORKSPACE needs VT_BWD_OVERWRITE and the workspace");
    if (st != VT_OK) return st;
    VT_REQUIRE(diffuse && specular, "vt_trace_bwd: null textures");
    VT_REQUIRE(num_rays == 0 || (rgba && rgba_grad), "vt_trace_bwd: null rgba inputs");
    VT_REQUIRE(points_grad && diffuse_grad && specular_grad && density_grad,
               "vt_trace_bwd: null gradient outputs");
    VT_REQUIRE(num_quantiles == 0 || (quantile_indices && depth_grad),
               "vt_trace_bwd: depth_grad must be provided if depth_quantiles is provided");
    if (num_rays == 0) {
        if (!overwrite) return VT_OK;
        // nothing to add: overwriting means zero gradients
        const size_t n = scene->num_points, at = attr_half ? 2 : 4;
        cudaStream_t s0 = (cudaStream_t)stream;
        cudaError_t e = cudaMemsetAsync(points_grad, 0, n * 12, s0);
        if (e == cudaSuccess) e = cudaMemsetAsync(diffuse_grad, 0, n * 3 * res * res * at, s0);
        if (e == cudaSuccess) e = cudaMemsetAsync(specular_grad, 0, n * 3 * res * res * at, s0);
        if (e == cudaSuccess) e = cudaMemsetAsync(density_grad, 0, n * 4, s0);
        if (e == cudaSuccess && point_error) e = cudaMemsetAsync(point_error, 0, n * at, s0);
        if (e != cudaSuccess) return vt::set_error(VT_ERR_CUDA, "vt_trace_bwd: %s", cudaGetErrorString(e));
        return VT_OK;
    }
    vt::PathRec rec{nullptr, 0, 0, nullptr};
    if (path && path->steps && path->cap) {
        VT_REQUIRE(path->len, "vt_trace_bwd: path record without len");
        VT_REQUIRE(((uintptr_t)path->steps & 15u) == 0, "vt_trace_bwd: path steps must be 16-byte aligned");
        rec = vt::PathRec{(uint4 *)path->steps, path->cap, num_rays, path->len};
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (attr_half) {
        vt::BwdIn<__half> b{quantile_indices, (const __half *)rgba, (const __half *)rgba_grad,
                            depth_grad, (const __half *)ray_error, contribution_alpha_grad,
                            distortion, distortion_grad, W_total, S_total, points_grad,
                            (__half *)diffuse_grad, (__half *)specular_grad, density_grad,
                            (__half *)point_error};
        b.rec = rec;
        if (res == 8)
            return vt::launch_bwd<__half, 8>(a, diffuse, specular, b, workspace, overwrite, keep_ws, s);
        if (res == 4)
            return vt::launch_bwd<__half, 4>(a, diffuse, specular, b, workspace, overwrite, keep_ws, s);
    } else {
        vt::BwdIn<float> b{quantile_indices, (const float *)rgba, (const float *)rgba_grad,
                           depth_grad, (const float *)ray_error, contribution_alpha_grad,
                           distortion, distortion_grad, W_total, S_total, points_grad,
                           (float *)diffuse_grad, (float *)specular_grad, density_grad,
                           (float *)point_error};
        b.rec = rec;
        if (res == 8)
            return vt::launch_bwd<float, 8>(a, diffuse, specular, b, workspace, overwrite, keep_ws, s);
        if (res == 4)
            return vt::launch_bwd<float, 4>(a, diffuse, specular, b, workspace, overwrite, keep_ws, s);
    }
    return vt::set_error(VT_ERR_INVALID, "vt_trace_bwd: res must be 4 or 8, got %d", res);
}
