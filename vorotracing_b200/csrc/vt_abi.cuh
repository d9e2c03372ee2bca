// vt_abi.cuh -- error plumbing shared by the extern "C" entry points.
// No exception ever crosses the C ABI: failures set a thread-local message
// and return a vt_status.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/vorotracing_b200.h"

namespace vt {

vt_status set_error(vt_status code, const char *fmt, ...);

inline vt_status check_launch(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(VT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return VT_OK;
}

inline unsigned grid_for(uint64_t n, unsigned block)
{
    return (unsigned)((n + block - 1) / block);
}

// Device-side data error reporting: first error wins.
__device__ __forceinline__ void report(uint32_t *err, uint32_t code)
{
    if (err) atomicCAS(err, 0u, code);
}

}  // namespace vt

#define VT_REQUIRE(cond, ...)                                                                     \
    do {                                                                                          \
        if (!(cond)) return vt::set_error(VT_ERR_INVALID, __VA_ARGS__);                           \
    } while (0)
