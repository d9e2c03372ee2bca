/*
 * vto_math.h -- TEST INFRASTRUCTURE (CPU oracle). Not part of the product.
 *
 * Exactly specified scalar primitives shared in *definition* (not in code)
 * with the CUDA kernels in vorotracing_b200/csrc/vt_math.cuh.  Both sides
 * evaluate the same sequence of IEEE-754 binary32 operations (round to
 * nearest even, no FMA contraction except where fmaf() is written out, no
 * flush-to-zero), so traversal decisions and colours agree bit for bit.
 *
 *  vto_expf: Cody & Waite range reduction x = k*ln2 + r, |r| <= ~0.35,
 *            e^r by its degree-7 Taylor polynomial (coefficients 1/n!),
 *            evaluated with Horner's rule in fmaf, then scaled by 2^k in two
 *            exact power-of-two steps.  Error <= 2 ulp against exp() in
 *            binary64 (checked by tests/test_oracle_math.py).
 *  vto_logf: x = m*2^e with m in [sqrt(1/2), sqrt(2)); log(m) = 2*atanh(s),
 *            s = (m-1)/(m+1), by the odd series 2s(1 + s^2/3 + ... + s^10/11).
 *  vto_f2h / vto_h2f: binary32 <-> binary16 with round-to-nearest-even.
 *
 * The reference uses CUDA's expf/logf built with -use_fast_math
 * (vorotracing/cuda/_backend.py:188-204); those are not reproducible on a CPU,
 * so parity with the reference binary itself is unpinned at this boundary.
 */
#ifndef VTO_MATH_H
#define VTO_MATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float vto_bits2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t vto_f2bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* ln2 split into a 24-bit head and a tail; 1/n! rounded to binary32. */
#define VTO_LOG2E   1.44269504088896341f
#define VTO_LN2_HI  0.693147182464599609375f
#define VTO_LN2_LO  -1.904654323148236e-09f

static inline float vto_pow2i(int k) /* 2^k, k in [-126, 127] */
{
    return vto_bits2f((uint32_t)(k + 127) << 23);
}

static inline float vto_expf(float x)
{
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    float kf = rintf(x * VTO_LOG2E);
    float r = fmaf(kf, -VTO_LN2_HI, x);
    r = fmaf(kf, -VTO_LN2_LO, r);
    float p = 1.98412698412698e-4f;           /* 1/7! */
    p = fmaf(p, r, 1.38888888888889e-3f);     /* 1/6! */
    p = fmaf(p, r, 8.33333333333333e-3f);     /* 1/5! */
    p = fmaf(p, r, 4.16666666666667e-2f);     /* 1/4! */
    p = fmaf(p, r, 1.66666666666667e-1f);     /* 1/3! */
    p = fmaf(p, r, 0.5f);                     /* 1/2! */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)kf;
    int k1 = k / 2;
    int k2 = k - k1;
    return (p * vto_pow2i(k1)) * vto_pow2i(k2);
}

static inline float vto_logf(float x)
{
    if (x != x) return x;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (x == INFINITY) return x;
    int e = 0;
    uint32_t u = vto_f2bits(x);
    if (u < 0x00800000u) { /* subnormal: scale into the normal range */
        x = x * 8388608.0f;
        u = vto_f2bits(x);
        e = -23;
    }
    e += (int)(u >> 23) - 127;
    float m = vto_bits2f((u & 0x007fffffu) | 0x3f800000u); /* [1, 2) */
    if (m > 1.41421353816986083984375f) {
        m = m * 0.5f;
        e += 1;
    }
    float f = m - 1.0f;
    float s = f / (2.0f + f);
    float z = s * s;
    float q = 9.09090909090909e-2f;           /* 1/11 */
    q = fmaf(q, z, 1.11111111111111e-1f);     /* 1/9 */
    q = fmaf(q, z, 1.42857142857143e-1f);     /* 1/7 */
    q = fmaf(q, z, 2.0e-1f);                  /* 1/5 */
    q = fmaf(q, z, 3.33333333333333e-1f);     /* 1/3 */
    float two_s = s + s;
    float lm = fmaf(two_s * z, q, two_s);     /* 2s + 2s*z*q */
    float ef = (float)e;
    return fmaf(ef, VTO_LN2_HI, fmaf(ef, VTO_LN2_LO, lm));
}

static inline float vto_h2f(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    if (ex == 0x1f) return vto_bits2f(sign | 0x7f800000u | (mant << 13));
    if (ex == 0) {
        float v = (float)mant * 5.9604644775390625e-8f; /* 2^-24, exact */
        return (h & 0x8000u) ? -v : v;
    }
    return vto_bits2f(sign | ((ex + 112u) << 23) | (mant << 13));
}

static inline uint16_t vto_f2h(float f)
{
    uint32_t x = vto_f2bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u);
    if (ax >= 0x477ff000u) return sign | 0x7c00u;
    if (ax >= 0x38800000u) {
        uint32_t r = (ax - 0x38000000u) + 0x0fffu + ((ax >> 13) & 1u);
        return sign | (uint16_t)(r >> 13);
    }
    float t = vto_bits2f(ax) * 16777216.0f; /* * 2^24, exact */
    return sign | (uint16_t)rintf(t);
}

#endif
