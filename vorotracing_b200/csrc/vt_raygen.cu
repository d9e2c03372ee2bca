// vt_raygen.cu -- camera ray generation on the GPU for the benchmark cameras.
//
// Pinhole rays follow the reference's generate_camera_rays convention
// (vorotracing/utils/__init__.py:85-130): integer pixel coordinates,
// x = (u - cx) / fx, y = (v - cy) / fy, camera direction (x, y, 1)
// normalised, rotated to world by the camera-to-world matrix and normalised
// again; origin = camera centre.  Further models (no reference counterpart,
// needed by the non-pinhole benchmark configuration):
//   equidistant fisheye  r = f * theta: direction (sin t * x/r, sin t * y/r, cos t), t = r
//   rolling shutter      row v is exposed at time v/(H-1) * duration and the
//                        centre moves linearly with `velocity` (world units / s)
//   thin lens            spp stratified samples per pixel on a lens disk of
//                        radius lens_radius (concentric square-to-disk map),
//                        focused at depth focus_distance along the optical axis
// Random numbers: Wellons' lowbias32 integer hash of (seed, pixel, sample,
// dimension), top 24 bits scaled to [0, 1).
#include "vt_abi.cuh"
#include "vt_geom.cuh"

namespace vt {

__device__ __forceinline__ uint32_t lowbias32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ float rand01(uint32_t seed, uint32_t pix, uint32_t s, uint32_t dim)
{
    uint32_t h = lowbias32(seed ^ lowbias32(pix ^ lowbias32(s * 4u + dim)));
    return (float)(h >> 8) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ V3 rot(const float *M, V3 v)  // 3x4 row-major, rotation part
{
    return mk(fmaf(M[2], v.z, fmaf(M[1], v.y, M[0] * v.x)),
              fmaf(M[6], v.z, fmaf(M[5], v.y, M[4] * v.x)),
              fmaf(M[10], v.z, fmaf(M[9], v.y, M[8] * v.x)));
}

__device__ __forceinline__ V3 unit(V3 v) { return divs(v, norm(v)); }

__global__ void raygen_kernel(vt_camera cam, float *__restrict__ rays)
{
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t total = (uint64_t)cam.width * cam.height * cam.spp;
    if (i >= total) return;
    uint32_t s = (uint32_t)(i % cam.spp);
    uint32_t pix = (uint32_t)(i / cam.spp);
    uint32_t u = pix % cam.width, v = pix / cam.width;
    float x = ((float)u - cam.K[2]) / cam.K[0];
    float y = ((float)v - cam.K[3]) / cam.K[1];
    V3 centre = mk(cam.c2w[3], cam.c2w[7], cam.c2w[11]);
    V3 o = centre, dc;
    switch (cam.model) {
    case VT_CAMERA_FISHEYE: {
        float r = sqrtf(fmaf(y, y, x * x));
        if (r > 0.0f) {
            float st = sinf(r), ct = cosf(r);
            dc = mk(st * (x / r), st * (y / r), ct);
        } else {
            dc = mk(0.0f, 0.0f, 1.0f);
        }
        break;
    }
    case VT_CAMERA_ROLLING: {
        dc = unit(mk(x, y, 1.0f));
        float t = cam.height > 1 ? (float)v / (float)(cam.height - 1) * cam.rs_duration : 0.0f;
        o = fma3(mk(cam.velocity[0], cam.velocity[1], cam.velocity[2]), t, centre);
        break;
    }
    case VT_CAMERA_THIN_LENS: {
        uint32_t g = 1;
        while (g * g < cam.spp) ++g;
        float a = ((float)(s % g) + rand01(cam.seed, pix, s, 0)) / (float)g * 2.0f - 1.0f;
        float b = ((float)(s / g) + rand01(cam.seed, pix, s, 1)) / (float)g * 2.0f - 1.0f;
        float lx = 0.0f, ly = 0.0f;
        if (a != 0.0f || b != 0.0f) {  // Shirley-Chiu concentric map
            float rr, phi;
            if (fabsf(a) > fabsf(b)) {
                rr = a;
                phi = 0.78539816339744831f * (b / a);
            } else {
                rr = b;
                phi = 1.5707963267948966f - 0.78539816339744831f * (a / b);
            }
            lx = cam.lens_radius * rr * cosf(phi);
            ly = cam.lens_radius * rr * sinf(phi);
        }
        V3 focus = mk(x * cam.focus_distance, y * cam.focus_distance, cam.focus_distance);
        V3 lens = mk(lx, ly, 0.0f);
        dc = unit(focus - lens);
        o = centre + rot(cam.c2w, lens);
        break;
    }
    default:
        dc = unit(mk(x, y, 1.0f));
    }
    V3 d = unit(rot(cam.c2w, dc));
    float *out = rays + i * 6;
    out[0] = o.x;
    out[1] = o.y;
    out[2] = o.z;
    out[3] = d.x;
    out[4] = d.y;
    out[5] = d.z;
}

}  // namespace vt

extern "C" vt_status vt_raygen(const vt_camera *cam, float *rays, vt_stream stream)
{
    VT_REQUIRE(cam && rays, "vt_raygen: null pointer");
    VT_REQUIRE(cam->spp >= 1, "vt_raygen: spp must be >= 1");
    VT_REQUIRE(cam->model >= VT_CAMERA_PINHOLE && cam->model <= VT_CAMERA_THIN_LENS,
               "vt_raygen: unknown camera model %d", cam->model);
    VT_REQUIRE(cam->K[0] != 0.0f && cam->K[1] != 0.0f, "vt_raygen: zero focal length");
    uint64_t total = (uint64_t)cam->width * cam->height * cam->spp;
    if (total == 0) return VT_OK;
    vt::raygen_kernel<<<vt::grid_for(total, 256), 256, 0, (cudaStream_t)stream>>>(*cam, rays);
    return vt::check_launch("vt_raygen");
}
