// status.cu — status codes and per-thread error detail for the C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace ofb {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char *what) {
    set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? OFB_ENOMEM : OFB_ECUDA;
}

constexpr int kMaxDev = 64;

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) dev = 0;
    return dev;
}

int sm_count() {
    static int n[kMaxDev];
    const int dev = current_device();
    if (!n[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n[dev] = v > 0 ? v : 148;
    }
    return n[dev];
}

}  // namespace ofb

extern "C" const char *ofb_last_error(void) { return ofb::g_err; }

extern "C" const char *ofb_status_string(int s) {
    switch (s) {
    case OFB_OK: return "ok";
    case OFB_EINVAL: return "invalid argument";
    case OFB_ECUDA: return "CUDA error";
    case OFB_ENOMEM: return "out of device memory";
    case OFB_EUNSUPPORTED: return "unsupported shape or mode";
    case OFB_ETOOLARGE: return "request exceeds capacity";
    default: return "unknown status";
    }
}

extern "C" const char *ofb_build_info(void) {
    return "ornith-flight-b200: sm_100a kernels, CUDA " OFB_STR(__CUDACC_VER_MAJOR__) "." OFB_STR(
        __CUDACC_VER_MINOR__);
}
