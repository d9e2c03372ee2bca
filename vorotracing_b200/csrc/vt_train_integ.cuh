// vt_train_integ.cuh -- training integrators (fp32 or fp16 attributes, layout
// (N, 3*R*R) with texel t channel c at t*3 + c).
//
//   FwdInteg  ray_integrator_octmap.cuh:57-282: colour only for density > 1e-6
//             but T always advances; mip-NeRF 360 distortion accumulators in
//             s = 1 - 1/(1+t) space; optional per-cell contribution; depth at
//             the transmittance quantiles; continue while T > weight_threshold.
//   BwdInteg  ray_integrator_octmap.cuh:635-1027: replays the forward and
//             scatters gradients; site gradients through the bisector-plane
//             geometry are flushed one cell late; the walk stops (and flushes
//             the pending site gradient) only when T < weight_threshold.
#pragma once

#include "vt_geom.cuh"

namespace vt {

template <class AT> __device__ __forceinline__ float tof(AT v);
template <> __device__ __forceinline__ float tof<float>(float v) { return v; }
template <> __device__ __forceinline__ float tof<__half>(__half v) { return __half2float(v); }
template <class AT> __device__ __forceinline__ AT fromf(float v);
template <> __device__ __forceinline__ float fromf<float>(float v) { return v; }
template <> __device__ __forceinline__ __half fromf<__half>(float v) { return __float2half_rn(v); }

template <class AT> __device__ __forceinline__ void atomic_add(AT *p, float v);
template <> __device__ __forceinline__ void atomic_add<float>(float *p, float v) { atomicAdd(p, v); }
template <> __device__ __forceinline__ void atomic_add<__half>(__half *p, float v)
{
    atomicAdd(p, __float2half_rn(v));
}

template <class AT, int R> struct TexPlain {
    const AT *diffuse;
    const AT *specular;
    __device__ __forceinline__ V3 logits(uint32_t cell, const Bilin &d, const Bilin &s) const
    {
        const AT *dp = diffuse + (size_t)cell * (3 * R * R);
        const AT *sp = specular + (size_t)cell * (3 * R * R);
        float a[4][3], b[4][3];
        const int di[4] = {d.i00, d.i10, d.i01, d.i11};
        const int si[4] = {s.i00, s.i10, s.i01, s.i11};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                a[k][c] = tof<AT>(dp[di[k] * 3 + c]);
                b[k][c] = tof<AT>(sp[si[k] * 3 + c]);
            }
        float r[3];
#pragma unroll
        for (int c = 0; c < 3; ++c)
            r[c] = blend(d, a[0][c], a[1][c], a[2][c], a[3][c]) +
                   blend(s, b[0][c], b[1][c], b[2][c], b[3][c]);
        return mk(r[0], r[1], r[2]);
    }
};

template <class AT, int R> struct FwdInteg {
    Ray ray;
    TexPlain<AT, R> tex;
    Bilin spec;
    float wt;
    V3 acc;
    float T;
    uint32_t ntex;
    const float *qthr;
    uint32_t K, qi;
    float qv;
    float *qdepth;
    uint32_t *qidx;
    float W, S, dist, self, tfar;
    float s_prev;  // 1 - 1/(1 + t0) of the current t0 (the previous segment's s1)
    AT *contrib;
    V3 last_rgb;   // colour of the last integrated segment (for the path record)

    __device__ __forceinline__ FwdInteg(const Ray &r, const TexPlain<AT, R> &t, float wt_,
                                        const float *qthr_, uint32_t K_, float *qdepth_,
                                        uint32_t *qidx_, AT *contrib_)
        : ray(r), tex(t), wt(wt_), acc(mk(0.f, 0.f, 0.f)), T(1.0f), ntex(0), qthr(qthr_), K(K_),
          qi(0), qv(0.0f), qdepth(qdepth_), qidx(qidx_), W(0.f), S(0.f), dist(0.f), self(0.f),
          tfar(0.f), s_prev(0.f), contrib(contrib_)
    {
        if (K > 0) qv = qthr[0];
        float tu, tv;
        oct_encode<R>(mk(-r.d.x, -r.d.y, -r.d.z), tu, tv);
        spec = make_bilin<R>(tu, tv);
    }

    __device__ __forceinline__ uint32_t textured() const { return ntex; }

    __device__ __forceinline__ bool integrate(uint32_t cell, float t0, float t1, V3 P, V3, float s)
    {
        V3 rgb = mk(0.f, 0.f, 0.f);
        if (s > 1e-6f) {
            float tu, tv;
            oct_encode<R>(probe_dir(ray, t0, P), tu, tv);
            Bilin d = make_bilin<R>(tu, tv);
            V3 l = tex.logits(cell, d, spec);
            rgb = mk(sigmoid(l.x), sigmoid(l.y), sigmoid(l.z));
            ntex++;
        }
        last_rgb = rgb;
        float delta = fmaxf(t1 - t0, 0.0f);
        float alpha = 1.0f - expf_exact(-s * delta);
        float w = T * alpha;
        // the walk integrates [t0, t1] only for t1 > t0 and then sets t0 = t1,
        // so this segment's t0 is the previous one's t1 (0 before the first)
        // and its s value was already computed: 1 - 1/(1 + 0) = 0 to start
        float s0 = s_prev;
        float s1 = 1.0f - 1.0f / (1.0f + t1);
        s_prev = s1;
        float mid = 0.5f * (s0 + s1);
        float ds = s1 - s0;
        dist = fmaf(w, fmaf(mid, W, -S), dist);
        self = fmaf(w * w, ds, self);
        W += w;
        S = fmaf(w, mid, S);
        if (t1 > tfar) tfar = t1;
        if (contrib) atomic_add<AT>(contrib + cell, w);
        acc = fma3(rgb, w, acc);
        float nT = T * (1.0f - alpha);
        while (qi < K && nT < qv) {
            qdepth[qi] = t0 + logf_exact(T / qv) / s;
            qidx[qi] = cell;
            qi++;
            if (qi < K) qv = qthr[qi];
        }
        T = nT;
        return T > wt;
    }
};

// d t / d site for the bisector-plane hit (ray_integrator.cuh:39-53).
__device__ __forceinline__ V3 cig(V3 p, V3 q, const Ray &ray)
{
    V3 fo = 0.5f * (p + q);
    V3 n = q - p;
    float num = dot(fo - ray.o, n);
    float dp = dot(n, ray.d);
    V3 g = num * ray.d + dp * (ray.o - p);
    return divs(g, dp * dp);
}

__device__ __forceinline__ void atomic_add3(float *p, V3 v)
{
    atomicAdd(p, v.x);
    atomicAdd(p + 1, v.y);
    atomicAdd(p + 2, v.z);
}

// Feature switches of the backward (compile time): the common training step
// has none of them, and their per-ray state then costs no registers.
constexpr int kBwdDepth = 1;  // depth-quantile gradients
constexpr int kBwdDist = 2;   // distortion-loss gradient
constexpr int kBwdErr = 4;    // per-cell point_error accumulation

template <class AT, int R, int F = kBwdDepth | kBwdDist | kBwdErr> struct BwdInteg {
    Ray ray;
    TexPlain<AT, R> tex;
    Bilin spec;
    float wt;
    V3 acc;
    float T;
    uint32_t ntex;
    V3 fwd_rgb, g_rgb;
    float fwd_a, g_a;
    const float *qthr;
    const float *dgrad;
    uint32_t K, qi;
    float qv, cur_dg, ray_error;
    float W, S, Wt, St, dgr, Dt, Drun;
    float s_prev;
    float *pgrad;
    AT *ddiff, *dspec;
    // Optional padded fp32 scratch: one float4 per texel / site, accumulated
    // with vector atomics (1 instead of 3 per texel); null = scalar atomics
    // straight into the outputs.
    float4 *sdiff, *sspec, *spts;
    float *sperr;  // fp32 point_error scratch (with the padded scratch), else null
    float *dden;
    AT *perr;
    V3 prev_geom, prev_grad, cur_grad, next_grad;
    uint32_t prev_idx;
    // This warp's 32 staging slots in shared memory (texel aggregation).
    struct AggLane {
        float4 wd, ws, dl;
    };
    AggLane *agg;

    __device__ __forceinline__ uint32_t textured() const { return ntex; }

    // Both texel scatters of a textured segment with warp aggregation.  A
    // warp's rays are neighbouring pixels that enter the same cells at the
    // same step (about 3 lanes per distinct cell on C2) with nearly equal
    // specular and often equal diffuse footprints, so lanes scattering into
    // the same cell with the same four texels (matched among the converged
    // lanes) sum their weighted contributions first and the group's lowest
    // lane issues the four float4 reductions.  The sums go through shared
    // memory: every lane of a group stages its weights and its dl in its
    // slot, and each group's leader adds its members' terms in lane order.
    // All groups of the warp are summed at once by their leaders (a shuffle
    // loop would run once per group, the groups one after another).
    __device__ __forceinline__ static unsigned long long footprint_key(uint32_t cell,
                                                                       const Bilin &b)
    {
        return ((unsigned long long)cell << 32) |
               (uint32_t)((b.i00 & 0xff) | (b.i10 & 0xff) << 8 | (b.i01 & 0xff) << 16 |
                          (b.i11 & 0xff) << 24);
    }

    template <bool kSpec>
    __device__ __forceinline__ void leader_scatter4(float4 *g, uint32_t cell, const Bilin &b,
                                                    V3 dl, unsigned grp) const
    {
        float4 s00 = make_float4(b.w00 * dl.x, b.w00 * dl.y, b.w00 * dl.z, 0.0f);
        float4 s10 = make_float4(b.w10 * dl.x, b.w10 * dl.y, b.w10 * dl.z, 0.0f);
        float4 s01 = make_float4(b.w01 * dl.x, b.w01 * dl.y, b.w01 * dl.z, 0.0f);
        float4 s11 = make_float4(b.w11 * dl.x, b.w11 * dl.y, b.w11 * dl.z, 0.0f);
        for (unsigned m = grp & (grp - 1); m; m &= m - 1) {
            const AggLane &o = agg[__ffs(m) - 1];
            const float4 w = kSpec ? o.ws : o.wd;
            const float4 d = o.dl;
            s00.x += w.x * d.x; s00.y += w.x * d.y; s00.z += w.x * d.z;
            s10.x += w.y * d.x; s10.y += w.y * d.y; s10.z += w.y * d.z;
            s01.x += w.z * d.x; s01.y += w.z * d.y; s01.z += w.z * d.z;
            s11.x += w.w * d.x; s11.y += w.w * d.y; s11.z += w.w * d.z;
        }
        float4 *base = g + (size_t)cell * (R * R);
        atomicAdd(base + b.i00, s00);
        atomicAdd(base + b.i10, s10);
        atomicAdd(base + b.i01, s01);
        atomicAdd(base + b.i11, s11);
    }

    __device__ __forceinline__ void scatter_grouped(uint32_t cell, const Bilin &bd, V3 dl) const
    {
        const unsigned act = __activemask();
        const unsigned me = 1u << (threadIdx.x & 31);
        const unsigned gd = __match_any_sync(act, footprint_key(cell, bd));
        const unsigned gs = __match_any_sync(act, footprint_key(cell, spec));
        if ((gd | gs) != me) {
            AggLane &o = agg[threadIdx.x & 31];
            o.wd = make_float4(bd.w00, bd.w10, bd.w01, bd.w11);
            o.ws = make_float4(spec.w00, spec.w10, spec.w01, spec.w11);
            o.dl = make_float4(dl.x, dl.y, dl.z, 0.0f);
        }
        __syncwarp(act);
        if ((gd & (me - 1)) == 0) leader_scatter4<false>(sdiff, cell, bd, dl, gd);
        if ((gs & (me - 1)) == 0) leader_scatter4<true>(sspec, cell, spec, dl, gs);
        __syncwarp(act);  // the slots are written again at the next segment
    }

    __device__ __forceinline__ void add_site(uint32_t idx, V3 v) const
    {
        if (spts)
            atomicAdd(spts + idx, make_float4(v.x, v.y, v.z, 0.0f));
        else
            atomic_add3(pgrad + (size_t)idx * 3, v);
    }

    __device__ __forceinline__ void scatter(AT *g, uint32_t cell, const Bilin &b, V3 dl) const
    {
        AT *base = g + (size_t)cell * (3 * R * R);
        const float d[3] = {dl.x, dl.y, dl.z};
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            atomic_add<AT>(base + b.i00 * 3 + c, b.w00 * d[c]);
            atomic_add<AT>(base + b.i10 * 3 + c, b.w10 * d[c]);
            atomic_add<AT>(base + b.i01 * 3 + c, b.w01 * d[c]);
            atomic_add<AT>(base + b.i11 * 3 + c, b.w11 * d[c]);
        }
    }

    __device__ __forceinline__ bool integrate(uint32_t cell, float t0, float t1, V3 P, V3 Q, float s)
    {
        return integrate_impl<false>(cell, t0, t1, P, Q, s, mk(0.f, 0.f, 0.f));
    }

    // The same with the segment's colour taken from the forward's path
    // record instead of re-sampling the texels (the forward computed it with
    // this very arithmetic, so the values are identical).
    __device__ __forceinline__ bool integrate_recorded(uint32_t cell, float t0, float t1, V3 P,
                                                       V3 Q, float s, V3 rgb_fwd)
    {
        return integrate_impl<true>(cell, t0, t1, P, Q, s, rgb_fwd);
    }

    template <bool kRecorded>
    __device__ __forceinline__ bool integrate_impl(uint32_t cell, float t0, float t1, V3 P, V3 Q,
                                                   float s, V3 rgb_fwd)
    {
        V3 rgb = mk(0.f, 0.f, 0.f);
        Bilin db;
        bool has_color = false;
        if (s > 1e-6f) {
            float tu, tv;
            oct_encode<R>(probe_dir(ray, t0, P), tu, tv);
            db = make_bilin<R>(tu, tv);
            if (kRecorded) {
                rgb = rgb_fwd;
            } else {
                V3 l = tex.logits(cell, db, spec);
                rgb = mk(sigmoid(l.x), sigmoid(l.y), sigmoid(l.z));
            }
            has_color = true;
            ntex++;
        }
        float delta = fmaxf(t1 - t0, 0.0f);
        float alpha = 1.0f - expf_exact(-s * delta);
        float w = T * alpha;
        float dads = delta * (1.0f - alpha);
        float dadd = 0.0f;
        if (delta > 0.0f) dadd = s * (1.0f - alpha);
        acc = acc + w * rgb;
        if constexpr ((F & kBwdErr) != 0)
            if (sperr)
                atomicAdd(sperr + cell, w * ray_error);
            else if (perr)
                atomic_add<AT>(perr + cell, w * ray_error);
        V3 dLdrgb = mk(g_rgb.x * w, g_rgb.y * w, g_rgb.z * w);
        V3 rest = divs(fwd_rgb - acc, T * ((1.0f - alpha) + 1e-6f));
        float dLda = T * dot(rgb - rest, g_rgb);
        dLda += ((1.0f - fwd_a) * g_a) / ((1.0f - alpha) + 1e-6f);
        float dLds = dLda * dads;
        float dLddt = dLda * dadd;
        float dLdt0 = 0.0f;
        if ((F & kBwdDist) != 0 && dgr != 0.0f) {
            float s0 = s_prev;  // as in FwdInteg: the previous segment's s1
            float s1 = 1.0f - 1.0f / (1.0f + t1);
            s_prev = s1;
            float mid = 0.5f * (s0 + s1);
            float ds = s1 - s0;
            float Wm = W, Sm = S;
            float Wp = (Wt - Wm) - w;
            float Sp = (St - Sm) - w * mid;
            float raw = (2.0f * (mid * Wm - Sm) + 2.0f * (Sp - mid * Wp)) + ((2.0f / 3.0f) * w) * ds;
            float outer = raw * dgr;
            float ww = outer * w;
            float Dip = (Dt - Drun) - ww;
            dLds += ((outer * T) * dads) - delta * Dip;
            Drun += ww;
            W += w;
            S += w * mid;
        }
        float nT = T * (1.0f - alpha);
        while ((F & kBwdDepth) != 0 && qi < K && nT < qv) {
            float gi = dgrad[qi] / s;
            dLdt0 += gi;
            dLds += ((-gi) * logf_exact(T / qv)) / s;
            cur_dg -= gi;
            qi++;
            if (qi < K) qv = qthr[qi];
        }
        if ((F & kBwdDepth) != 0 && qi < K) {
            dLds += (-delta) * cur_dg;
            dLddt += (-s) * cur_dg;
        }
        dLdt0 += -dLddt;
        float dLdt1 = dLddt;
        V3 g_prev = mk(0.f, 0.f, 0.f);
        if (prev_idx != 0xffffffffu) g_prev = cig(prev_geom, P, ray);
        V3 g1c = cig(P, Q, ray);
        V3 g0c = cig(P, prev_geom, ray);
        V3 g1n = cig(Q, P, ray);
        prev_grad = prev_grad + dLdt0 * g_prev;
        cur_grad = cur_grad + (dLdt0 * g0c + dLdt1 * g1c);
        next_grad = next_grad + dLdt1 * g1n;
        if (prev_idx != 0xffffffffu) add_site(prev_idx, prev_grad);
        prev_geom = P;
        prev_idx = cell;
        prev_grad = cur_grad;
        cur_grad = next_grad;
        next_grad = mk(0.f, 0.f, 0.f);
        T = nT;
        if (has_color) {
            V3 dl = mk((dLdrgb.x * rgb.x) * (1.0f - rgb.x), (dLdrgb.y * rgb.y) * (1.0f - rgb.y),
                       (dLdrgb.z * rgb.z) * (1.0f - rgb.z));
            if (sdiff) {
                scatter_grouped(cell, db, dl);
            } else {
                scatter(ddiff, cell, db, dl);
                scatter(dspec, cell, spec, dl);
            }
        }
        atomicAdd(dden + cell, dLds);
        if (T < wt) {
            add_site(prev_idx, prev_grad);
            return false;
        }
        return true;
    }
};

}  // namespace vt
