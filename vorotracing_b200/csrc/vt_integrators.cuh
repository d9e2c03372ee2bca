// vt_integrators.cuh -- per-cell segment integrators for the inference paths.
//
//   InferInteg<R, Tex>   ray_integrator_octmap.cuh:295-461 (fp16, Half4Texel)
//                        and :463-633 (q8, one global scale/offset per map).
// Density gate first (a cell with density <= 1e-6 leaves T untouched), colour
// only when the segment weight reaches cell_skip_threshold, T always advances
// otherwise, continue while T > weight_threshold.
#pragma once

#include "vt_geom.cuh"

namespace vt {

// Texture fetchers: colour logits of one cell for a bilinear footprint.
// All eight texel loads (4 diffuse + 4 specular) are issued before any use.
template <int R> struct TexF16x4 {
    const uint2 *diffuse;   // (N, R*R) Half4Texel rows, 8 bytes per texel
    const uint2 *specular;
    __device__ __forceinline__ V3 logits(uint32_t cell, const Bilin &d, const Bilin &s) const
    {
        const uint2 *dp = diffuse + (size_t)cell * (R * R);
        const uint2 *sp = specular + (size_t)cell * (R * R);
        uint2 a00 = __ldg(dp + d.i00), a10 = __ldg(dp + d.i10), a01 = __ldg(dp + d.i01),
              a11 = __ldg(dp + d.i11);
        uint2 b00 = __ldg(sp + s.i00), b10 = __ldg(sp + s.i10), b01 = __ldg(sp + s.i01),
              b11 = __ldg(sp + s.i11);
        auto lo = [](uint2 t) { return h2f((uint16_t)(t.x & 0xffffu)); };
        auto mid = [](uint2 t) { return h2f((uint16_t)(t.x >> 16)); };
        auto hi = [](uint2 t) { return h2f((uint16_t)(t.y & 0xffffu)); };
        V3 df = mk(blend(d, lo(a00), lo(a10), lo(a01), lo(a11)),
                   blend(d, mid(a00), mid(a10), mid(a01), mid(a11)),
                   blend(d, hi(a00), hi(a10), hi(a01), hi(a11)));
        V3 sf = mk(blend(s, lo(b00), lo(b10), lo(b01), lo(b11)),
                   blend(s, mid(b00), mid(b10), mid(b01), mid(b11)),
                   blend(s, hi(b00), hi(b10), hi(b01), hi(b11)));
        return df + sf;
    }
};

template <int R> struct TexQ8 {
    const uint8_t *diffuse;  // (N, 3*R*R) bytes
    const uint8_t *specular;
    float dscale, doffset, sscale, soffset;
    __device__ __forceinline__ V3 logits(uint32_t cell, const Bilin &d, const Bilin &s) const
    {
        const uint8_t *dp = diffuse + (size_t)cell * (3 * R * R);
        const uint8_t *sp = specular + (size_t)cell * (3 * R * R);
        uint8_t a[4][3], b[4][3];
        const int di[4] = {d.i00, d.i10, d.i01, d.i11};
        const int si[4] = {s.i00, s.i10, s.i01, s.i11};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                a[k][c] = __ldg(dp + di[k] * 3 + c);
                b[k][c] = __ldg(sp + si[k] * 3 + c);
            }
        float r[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float dv[4], sv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                dv[k] = fmaf(dscale, (float)a[k][c], doffset);
                sv[k] = fmaf(sscale, (float)b[k][c], soffset);
            }
            r[c] = blend(d, dv[0], dv[1], dv[2], dv[3]) + blend(s, sv[0], sv[1], sv[2], sv[3]);
        }
        return mk(r[0], r[1], r[2]);
    }
};

// q8 texels widened to one 4-byte word each (bytes r, g, b, 0; vt_pad_u8x4):
// one 32-bit load per texel instead of three byte loads, same values.
template <int R> struct TexQ8x4 {
    const uint32_t *diffuse;  // (N, R*R) words
    const uint32_t *specular;
    float dscale, doffset, sscale, soffset;
    __device__ __forceinline__ V3 logits(uint32_t cell, const Bilin &d, const Bilin &s) const
    {
        const uint32_t *dp = diffuse + (size_t)cell * (R * R);
        const uint32_t *sp = specular + (size_t)cell * (R * R);
        const uint32_t a[4] = {__ldg(dp + d.i00), __ldg(dp + d.i10), __ldg(dp + d.i01),
                               __ldg(dp + d.i11)};
        const uint32_t b[4] = {__ldg(sp + s.i00), __ldg(sp + s.i10), __ldg(sp + s.i01),
                               __ldg(sp + s.i11)};
        float r[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float dv[4], sv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                dv[k] = fmaf(dscale, (float)((a[k] >> (8 * c)) & 0xffu), doffset);
                sv[k] = fmaf(sscale, (float)((b[k] >> (8 * c)) & 0xffu), soffset);
            }
            r[c] = blend(d, dv[0], dv[1], dv[2], dv[3]) + blend(s, sv[0], sv[1], sv[2], sv[3]);
        }
        return mk(r[0], r[1], r[2]);
    }
};

template <int R, class Tex> struct InferInteg {
    Ray ray;
    Tex tex;
    Bilin spec;
    float wt, skip;
    V3 acc;
    float T;
    uint32_t ntex;

    __device__ __forceinline__ InferInteg(const Ray &r, const Tex &t, float wt_, float skip_)
        : ray(r), tex(t), wt(wt_), skip(skip_), acc(mk(0.f, 0.f, 0.f)), T(1.0f), ntex(0)
    {
        float tu, tv;
        oct_encode<R>(mk(-r.d.x, -r.d.y, -r.d.z), tu, tv);
        spec = make_bilin<R>(tu, tv);
    }

    __device__ __forceinline__ uint32_t textured() const { return ntex; }

    __device__ __forceinline__ bool integrate(uint32_t cell, float t0, float t1, V3 P, V3, float s)
    {
        if (s <= 1e-6f) return T > wt;
        float delta = fmaxf(t1 - t0, 0.0f);
        float alpha = 1.0f - expf_exact(-s * delta);
        float w = T * alpha;
        if (w >= skip) {
            float tu, tv;
            oct_encode<R>(probe_dir(ray, t0, P), tu, tv);
            Bilin d = make_bilin<R>(tu, tv);
            V3 l = tex.logits(cell, d, spec);
            V3 rgb = mk(sigmoid(l.x), sigmoid(l.y), sigmoid(l.z));
            acc = fma3(rgb, w, acc);
            ntex++;
        }
        T = T * (1.0f - alpha);
        return T > wt;
    }
};

}  // namespace vt

namespace vt {

// Depth-only integrator: the training forward's transmittance and depth-
// quantile rule (ray_integrator_octmap.cuh:114-151: T advances in every
// segment, depth_k = t0 + log(T / q_k) / density when T first drops below
// q_k, continue while T > weight_threshold) without any colour work.  Used
// for the viewer's depth modes (vorotracing/viewer.py:414-433): it returns
// the first quantile's depth, or the mean of the positive quantile depths.
struct DepthInteg {
    const float *thr;  // K thresholds shared by all rays, decreasing
    uint32_t K, qi;
    float qv, wt, T, sum, first;
    uint32_t cnt;

    __device__ __forceinline__ DepthInteg(const float *thr_, uint32_t K_, float wt_)
        : thr(thr_), K(K_), qi(0), qv(K_ ? thr_[0] : 0.0f), wt(wt_), T(1.0f), sum(0.0f),
          first(-1.0f), cnt(0)
    {
    }

    __device__ __forceinline__ uint32_t textured() const { return 0; }

    __device__ __forceinline__ bool integrate(uint32_t, float t0, float t1, V3, V3, float s)
    {
        float delta = fmaxf(t1 - t0, 0.0f);
        float alpha = 1.0f - expf_exact(-s * delta);
        float nT = T * (1.0f - alpha);
        while (qi < K && nT < qv) {
            float d = t0 + logf_exact(T / qv) / s;
            if (qi == 0) first = d;
            if (d > 0.0f) {
                sum += d;
                cnt++;
            }
            qi++;
            if (qi < K) qv = thr[qi];
        }
        T = nT;
        return T > wt;
    }
};

}  // namespace vt
