// vt_geom.cuh -- vectors, octahedral texture addressing and the packed face
// record shared by every traversal kernel.  Operation order is part of the
// parity contract with the CPU oracle (see vt_math.cuh): the multiply-adds
// that nvcc contracts when compiling the reference's expressions are written
// as explicit fmaf (dot products, face origin, hit point, bilinear blends,
// octahedral texel coordinates); everything else is one IEEE op per operator.
#pragma once

#include "vt_math.cuh"

namespace vt {

struct V3 {
    float x, y, z;
};

__device__ __forceinline__ V3 mk(float x, float y, float z) { return V3{x, y, z}; }
__device__ __forceinline__ V3 operator+(V3 a, V3 b) { return mk(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ V3 operator-(V3 a, V3 b) { return mk(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ V3 operator*(float s, V3 a) { return mk(s * a.x, s * a.y, s * a.z); }
__device__ __forceinline__ V3 divs(V3 a, float s) { return mk(a.x / s, a.y / s, a.z / s); }
__device__ __forceinline__ float dot(V3 a, V3 b) { return fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)); }
// a * s + b per component, contracted
__device__ __forceinline__ V3 fma3(V3 a, float s, V3 b)
{
    return mk(fmaf(a.x, s, b.x), fmaf(a.y, s, b.y), fmaf(a.z, s, b.z));
}
__device__ __forceinline__ float norm(V3 a) { return sqrtf(dot(a, a)); }
__device__ __forceinline__ V3 ld3(const float *__restrict__ p)
{
    return mk(__ldg(p), __ldg(p + 1), __ldg(p + 2));
}

struct Ray {
    V3 o, d;  // d normalised
};

// Ray load + normalisation (tracing_octmap.cu:179-180).
__device__ __forceinline__ Ray load_ray(const float *__restrict__ rays, uint32_t r)
{
    const float2 *p = reinterpret_cast<const float2 *>(rays + (size_t)r * 6);
    float2 a = __ldg(p), b = __ldg(p + 1), c = __ldg(p + 2);
    Ray ray;
    ray.o = mk(a.x, a.y, b.x);
    V3 d = mk(b.y, c.x, c.y);
    ray.d = divs(d, norm(d));
    return ray;
}

// Octahedral encoding (ray_integrator_octmap.cuh:17-35).
template <int R> __device__ __forceinline__ void oct_encode(V3 dir, float &tu, float &tv)
{
    float l1 = (fabsf(dir.x) + fabsf(dir.y)) + fabsf(dir.z);
    float inv_l1 = 1.0f / fmaxf(l1, 1e-10f);
    float u = dir.x * inv_l1;
    float v = dir.y * inv_l1;
    if (dir.z < 0.0f) {
        float ou = (1.0f - fabsf(v)) * copysignf(1.0f, u);
        float ov = (1.0f - fabsf(u)) * copysignf(1.0f, v);
        u = ou;
        v = ov;
    }
    tu = fmaf(fmaf(u, 0.5f, 0.5f), (float)R, -0.5f);
    tv = fmaf(fmaf(v, 0.5f, 0.5f), (float)R, -0.5f);
}

// Octahedral mirror wrap of an out-of-range texel (ray_integrator_octmap.cuh:37-55).
template <int R> __device__ __forceinline__ int oct_wrap(int ut, int vt_)
{
    if (ut >= 0 && ut < R && vt_ >= 0 && vt_ < R) return vt_ * R + ut;
    int wu = ((ut % R) + R) % R;
    int wv = ((vt_ % R) + R) % R;
    int fu = abs(ut / R) + (ut < 0 ? 1 : 0);
    int fv = abs(vt_ / R) + (vt_ < 0 ? 1 : 0);
    if (((fu ^ fv) & 1) != 0) {
        wu = R - 1 - wu;
        wv = R - 1 - wv;
    }
    return wv * R + wu;
}

struct Bilin {
    int i00, i10, i01, i11;
    float w00, w10, w01, w11;
};

template <int R> __device__ __forceinline__ Bilin make_bilin(float u, float v)
{
    Bilin b;
    int u0 = (int)floorf(u), v0 = (int)floorf(v);
    float fu = u - (float)u0, fv = v - (float)v0;
    b.i00 = oct_wrap<R>(u0, v0);
    b.i10 = oct_wrap<R>(u0 + 1, v0);
    b.i01 = oct_wrap<R>(u0, v0 + 1);
    b.i11 = oct_wrap<R>(u0 + 1, v0 + 1);
    b.w00 = (1.0f - fu) * (1.0f - fv);
    b.w10 = fu * (1.0f - fv);
    b.w01 = (1.0f - fu) * fv;
    b.w11 = fu * fv;
    return b;
}

__device__ __forceinline__ float blend(const Bilin &b, float a00, float a10, float a01, float a11)
{
    return fmaf(b.w11, a11, fmaf(b.w01, a01, fmaf(b.w10, a10, b.w00 * a00)));
}

// Direction from the site to the entry point (ray_integrator_octmap.cuh:258-264).
__device__ __forceinline__ V3 probe_dir(const Ray &ray, float t0, V3 P)
{
    V3 hit = fma3(ray.d, t0, ray.o);
    V3 dd = hit - P;
    float len = norm(dd);
    if (len > 1e-8f) {
#ifdef VT_REF_FASTMATH
        return mk(dd.x / len, dd.y / len, dd.z / len);  // the reference's d /= len
#else
        float inv = 1.0f / len;
        return mk(dd.x * inv, dd.y * inv, dd.z * inv);
#endif
    }
    return ray.d;
}

// ---------------------------------------------------------------------------
// Packed face record: one 16-byte row per CSR entry e (same index as the
// reference's adjacency / adj_diff arrays), so a cell's faces are read with
// 128-bit loads and the winning face already carries everything the walk
// needs to issue the next cell's loads:
//   x = half(dx) | half(dy) << 16        offset to the neighbour site (RNE)
//   y = half(dz) | deg(neighbour) << 16
//   z = neighbour id
//   w = CSR begin of the neighbour's faces
// The half offsets are the values of the reference's adj_diff
// (tracing_octmap.cu:125-149).
// ---------------------------------------------------------------------------
constexpr uint32_t kFacePadRows = 4;
constexpr uint32_t kMaxDegree = 0xffff;

__device__ __forceinline__ uint16_t face_deg(uint4 f) { return (uint16_t)(f.y >> 16); }

}  // namespace vt
