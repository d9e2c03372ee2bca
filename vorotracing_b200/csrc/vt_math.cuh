// vt_math.cuh -- exactly specified scalar primitives for the traversal kernels.
//
// Every file that includes this header is compiled with -fmad=false and
// without --use_fast_math, so each binary32 +, -, *, / and sqrt is a single
// IEEE-754 round-to-nearest-even operation and no multiply-add is contracted
// unless fmaf() is written out.  The CPU oracle evaluates the same operation
// sequence, so traversal decisions and colours agree bit for bit.
//
//  vt_expf: Cody & Waite reduction x = k*ln2 + r, e^r by its degree-7 Taylor
//           polynomial (coefficients 1/n!) in Horner form, then exact scaling
//           by 2^k in two power-of-two steps (<= 1 ulp from exp in binary64).
//  vt_logf: x = m*2^e, m in [sqrt(1/2), sqrt(2)); log m = 2 atanh(s),
//           s = (m-1)/(m+1), odd series to s^11 (<= 2 ulp).
// The reference evaluates expf/logf under -use_fast_math
// (vorotracing/cuda/_backend.py:188-204), which has no portable definition.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace vt {

constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693147182464599609375f;
constexpr float kLn2Lo = -1.904654323148236e-09f;

__device__ __forceinline__ float pow2i(int k)  // 2^k for k in [-126, 127]
{
    return __int_as_float((k + 127) << 23);
}

#ifdef VT_REF_FASTMATH
// Measurement build only (libvorotracing_b200_refmath.so, never the product):
// the reference's arithmetic, compiled like vorotracing/cuda/_backend.py:188-204
// (-use_fast_math, contraction on), so that CUDA's fast expf / logf and
// approximate division stand where the reference has them.  Tests compare
// this build with the exact one to bound how far the reference binary's
// results can sit from the oracle's.
__device__ __forceinline__ float expf_exact(float x) { return expf(x); }
__device__ __forceinline__ float logf_exact(float x) { return logf(x); }
#else
__device__ __forceinline__ float expf_exact(float x)
{
    if (x != x) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.97208404541015625f) return 0.0f;
    float kf = rintf(x * kLog2e);
    float r = fmaf(kf, -kLn2Hi, x);
    r = fmaf(kf, -kLn2Lo, r);
    float p = 1.98412698412698e-4f;
    p = fmaf(p, r, 1.38888888888889e-3f);
    p = fmaf(p, r, 8.33333333333333e-3f);
    p = fmaf(p, r, 4.16666666666667e-2f);
    p = fmaf(p, r, 1.66666666666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)kf;
    int k1 = k / 2;
    int k2 = k - k1;
    return (p * pow2i(k1)) * pow2i(k2);
}

__device__ __forceinline__ float logf_exact(float x)
{
    if (x != x) return x;
    if (x < 0.0f) return __int_as_float(0x7fc00000);
    if (x == 0.0f) return __int_as_float(0xff800000);
    if (x == __int_as_float(0x7f800000)) return x;
    int e = 0;
    uint32_t u = __float_as_uint(x);
    if (u < 0x00800000u) {
        x = x * 8388608.0f;
        u = __float_as_uint(x);
        e = -23;
    }
    e += (int)(u >> 23) - 127;
    float m = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421353816986083984375f) {
        m = m * 0.5f;
        e += 1;
    }
    float f = m - 1.0f;
    float s = f / (2.0f + f);
    float z = s * s;
    float q = 9.09090909090909e-2f;
    q = fmaf(q, z, 1.11111111111111e-1f);
    q = fmaf(q, z, 1.42857142857143e-1f);
    q = fmaf(q, z, 2.0e-1f);
    q = fmaf(q, z, 3.33333333333333e-1f);
    float two_s = s + s;
    float lm = fmaf(two_s * z, q, two_s);
    float ef = (float)e;
    return fmaf(ef, kLn2Hi, fmaf(ef, kLn2Lo, lm));
}
#endif

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf_exact(-x)); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

}  // namespace vt
