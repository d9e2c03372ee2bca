// vt_abi.cu -- thread-local error state and version of the C ABI.
#include "vt_abi.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace vt {

vt_status set_error(vt_status code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

}  // namespace vt

extern "C" const char *vt_last_error(void) { return g_last_error; }

extern "C" const char *vt_version(void) { return "0.1.0"; }

extern "C" vt_status vt_host_device_ptr(const void *host, void **device)
{
    if (!host || !device) return vt::set_error(VT_ERR_INVALID, "vt_host_device_ptr: null pointer");
    void *d = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void *>(host), 0);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return vt::set_error(VT_ERR_INVALID, "vt_host_device_ptr: not mapped page-locked memory (%s)",
                             cudaGetErrorString(e));
    }
    *device = d;
    return VT_OK;
}
