// vt_optim.cu -- fused Adam step over the flat per-cell parameter layout.
//
// The reference trains the four per-cell parameter tensors with
// torch.optim.Adam(eps=1e-15, fused=...) in four learning-rate groups
// (vorotracing/trainer.py:503-527) and then clamps the log-density to <= 30
// (trainer.py:258-265).  Here parameters, gradients and both moments live in
// flat fp32 buffers laid out [points 3N | density N | diffuse | specular]
// (the gradient all-reduce bucket's layout), and one launch does the update
// of all four groups plus the clamp.  Per element, as torch's Adam:
//   m = m + (1 - b1) (g - m);  v = b2 v + (1 - b2) g^2
//   p -= (lr / (1 - b1^t)) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
#include "vt_abi.cuh"

namespace vt {

struct AdamArgs {
    uint64_t seg_end[4];  // exclusive end offsets of the four groups
    float lr[4];
    float beta1, beta2, eps;
    float bc1[4], bc2_sqrt;  // 1 - b1^t per group (same t), sqrt(1 - b2^t)
    int clamp_group;         // group whose values are clamped from above, -1 = none
    float clamp_max;
};

__global__ void adam_kernel(float *__restrict__ p, const float *__restrict__ g, float *__restrict__ m,
                            float *__restrict__ v, uint64_t n, AdamArgs a)
{
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        int grp = i < a.seg_end[0] ? 0 : i < a.seg_end[1] ? 1 : i < a.seg_end[2] ? 2 : 3;
        float gi = g[i];
        float mi = m[i];
        mi = fmaf(1.0f - a.beta1, gi - mi, mi);
        float vi = fmaf(a.beta2, v[i], (1.0f - a.beta2) * gi * gi);
        float denom = sqrtf(vi) / a.bc2_sqrt + a.eps;
        float pi = p[i] - (a.lr[grp] / a.bc1[grp]) * (mi / denom);
        if (grp == a.clamp_group) pi = fminf(pi, a.clamp_max);
        p[i] = pi;
        m[i] = mi;
        v[i] = vi;
    }
}

}  // namespace vt

extern "C" vt_status vt_adam_step(float *params, const float *grads, float *exp_avg,
                                  float *exp_avg_sq, uint64_t n, const uint64_t *group_ends,
                                  const float *lrs, float beta1, float beta2, float eps,
                                  uint32_t step, int clamp_group, float clamp_max,
                                  vt_stream stream)
{
    VT_REQUIRE(params && grads && exp_avg && exp_avg_sq && group_ends && lrs,
               "vt_adam_step: null pointer");
    VT_REQUIRE(step >= 1, "vt_adam_step: step counts from 1");
    VT_REQUIRE(group_ends[3] == n && group_ends[0] <= group_ends[1] &&
                   group_ends[1] <= group_ends[2] && group_ends[2] <= group_ends[3],
               "vt_adam_step: group ends must be non-decreasing and end at n");
    vt::AdamArgs a;
    for (int k = 0; k < 4; ++k) {
        a.seg_end[k] = group_ends[k];
        a.lr[k] = lrs[k];
        a.bc1[k] = (float)(1.0 - pow((double)beta1, (double)step));
    }
    a.beta1 = beta1;
    a.beta2 = beta2;
    a.eps = eps;
    a.bc2_sqrt = (float)sqrt(1.0 - pow((double)beta2, (double)step));
    a.clamp_group = clamp_group;
    a.clamp_max = clamp_max;
    if (n == 0) return VT_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    uint64_t want = (n + 255) / 256;
    unsigned grid = (unsigned)(want < (uint64_t)sms * 16 ? want : (uint64_t)sms * 16);
    vt::adam_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(params, grads, exp_avg, exp_avg_sq, n,
                                                            a);
    return vt::check_launch("adam_kernel");
}
