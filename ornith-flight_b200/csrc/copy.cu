// copy.cu — ofb_copy: a copy done by a kernel, for moving a decode step's
// activations between pinned host memory and the device. A copy-engine
// transfer of a few KB costs several microseconds of set-up and cannot
// overlap the kernel next to it; this kernel is launched with programmatic
// dependent launch like the layer kernels, reads or writes pinned host memory
// directly over the bus (unified addressing), and lets the next kernel start
// its own weight loads while it runs.
#include "common.cuh"

namespace ofb {

__global__ void __launch_bounds__(512) copy16_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                                     size_t n16) {
    pdl_wait();  // src may be the previous kernel's output
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

__global__ void __launch_bounds__(512) copy1_kernel(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src,
                                                    size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace ofb

using namespace ofb;

extern "C" int ofb_copy(void *dst, const void *src, size_t bytes, void *stream) {
    if (!bytes) return OFB_OK;
    if (!dst || !src) { set_error("ofb_copy: NULL pointer"); return OFB_EINVAL; }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0) {
        const size_t n16 = bytes / 16;
        e = launch_pdl(copy16_kernel, dim3(grid_for(n16, 512, 148 * 4)), dim3(512), 0, s,
                       static_cast<uint4 *>(dst), static_cast<const uint4 *>(src), n16);
    } else {
        e = launch_pdl(copy1_kernel, dim3(grid_for(bytes, 512, 148 * 4)), dim3(512), 0, s,
                       static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), bytes);
    }
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "ofb_copy launch");
}
