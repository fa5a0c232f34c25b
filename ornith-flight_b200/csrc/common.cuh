// common.cuh — shared device helpers: bit-exact K-quant field decode, error
// plumbing, warp reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ornith_moe.h"

#define OFB_STR2(x) #x
#define OFB_STR(x) OFB_STR2(x)

namespace ofb {

constexpr int QK = 256;
constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;

// Current device ordinal (0..63) and its SM count (cached per device).
int current_device();
int sm_count();

// Per-host-thread error detail (ofb_last_error).
void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

#define OFB_CHECK_LAUNCH(what)                                                  \
    do {                                                                        \
        cudaError_t e__ = cudaGetLastError();                                   \
        if (e__ != cudaSuccess) return ::ofb::cuda_status(e__, what);           \
    } while (0)

// fp16 bits -> f32 with the reference's rebias rule (engine/src/gguf.c:16-26):
// only 0x0000 maps to 0; every other pattern (subnormal, -0, exponent 31) is
// decoded as if it were a normal number.
__device__ __forceinline__ float half_bits_ref(uint32_t h) {
    if (h == 0) return 0.0f;
    uint32_t u = ((h & 0x8000u) << 16) | ((((h >> 10) & 0x1Fu) + 112u) << 23) | ((h & 0x3FFu) << 13);
    return __uint_as_float(u);
}

// 6-bit (scale, min) of Q4_K sub-block j from the 12 packed bytes held as
// three little-endian words s[0..2] (engine/src/gguf.c:31-40).
__device__ __forceinline__ void q4k_scale_min(const uint32_t s[3], int j, int &sc, int &mn) {
    // selects, not s[i >> 2]: a runtime index would put s in local memory
    auto byte = [&](int i) -> int {
        const uint32_t w = i < 4 ? s[0] : (i < 8 ? s[1] : s[2]);
        return (w >> (8 * (i & 3))) & 0xFF;
    };
    if (j < 4) {
        sc = byte(j) & 63;
        mn = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

// Reference rounding of one Q4_K element: (d*sc)*q - (dmin*m), every product
// rounded on its own (no contraction), engine/src/gguf.c:49-57.
__device__ __forceinline__ float q4k_value(float dsc, float dmm, int q) {
    return __fsub_rn(__fmul_rn(dsc, (float)q), dmm);
}

// Reference rounding of one Q6_K element: (d*sc)*q, engine/src/gguf.c:76-79.
__device__ __forceinline__ float q6k_value(float d, int sc, int q) {
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

// Single-element decode, used by the expert-slice entry point
// (engine/src/gguf.c:511-571); also the
// interleaved-layout MoE kernels.
__device__ __forceinline__ float q4k_one(const uint8_t *blk, int pos) {
    uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    int chunk = pos >> 6, hi = (pos >> 5) & 1;
    uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    int sc, mn;
    q4k_scale_min(s, 2 * chunk + hi, sc, mn);
    uint8_t byte = __ldg(blk + 16 + chunk * 32 + (pos & 31));
    int q = hi ? (byte >> 4) : (byte & 0xF);
    float dsc = __fmul_rn(half_bits_ref(hdr.x & 0xFFFFu), (float)sc);
    float dmm = __fmul_rn(half_bits_ref(hdr.x >> 16), (float)mn);
    return q4k_value(dsc, dmm, q);
}

__device__ __forceinline__ float q6k_one(const uint8_t *blk, int pos) {
    int half = pos >> 7, quad = (pos >> 5) & 3, l = pos & 31;
    uint8_t lo = __ldg(blk + half * 64 + (quad & 1) * 32 + l);
    int nib = (quad < 2) ? (lo & 0xF) : (lo >> 4);
    int top = (__ldg(blk + 128 + half * 32 + l) >> (2 * quad)) & 3;
    int q = (nib | (top << 4)) - 32;
    int sc = (int)(int8_t)__ldg(blk + 192 + half * 8 + quad * 2 + (l >> 4));
    float d = half_bits_ref((uint32_t)__ldg(blk + 208) | ((uint32_t)__ldg(blk + 209) << 8));
    return q6k_value(d, sc, q);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current
// device (function attributes are per device); `cache` remembers, per
// device, the largest value already set.
template <typename... KArgs>
inline cudaError_t ensure_dyn_smem(void (*kernel)(KArgs...), size_t bytes, size_t (&cache)[64]) {
    const int dev = current_device();
    if (bytes <= 48 * 1024 || bytes <= cache[dev]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) cache[dev] = bytes;
    return e;
}

inline int grid_for(uint64_t work, int per_block, int cap) {
    uint64_t g = (work + per_block - 1) / per_block;
    if (g > (uint64_t)cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace ofb

// ---- programmatic dependent launch (PDL) ----------------------------------
// A kernel launched with launch_pdl may start while the previous kernel in
// the stream is still running: it first does work that does not depend on
// that kernel (loading static weights), then pdl_wait() blocks until the
// previous grid has completed and its memory is visible. pdl_trigger() lets
// the next PDL kernel in the stream be scheduled early.
namespace ofb {
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// L2 prefetch of [p, p + bytes) spread over the calling threads.
// Optional launch timeline of the decode kernels (build with
// -DOFB_DECODE_TRACE): per launch, block 0 takes a ring slot and records
// globaltimer at start and after griddepcontrol.wait; every block raises the
// slot's end time. Each translation unit keeps its own ring (DTRACE_DEFINE).
#ifdef OFB_DECODE_TRACE
#define DTRACE_DEFINE(tag)                                                                        \
    __device__ unsigned long long g_dtr_##tag[4][64][6];                                          \
    __device__ unsigned int g_dtn_##tag[4], g_dtc_##tag[4];                                        \
    extern "C" int ofb_debug_dtrace_##tag(unsigned long long *host, int reset) {                   \
        if (reset) {                                                                              \
            static unsigned long long z[4 * 64 * 6];                                              \
            static unsigned int zn[4];                                                            \
            cudaMemcpyToSymbol(g_dtr_##tag, z, sizeof(z));                                        \
            return cudaMemcpyToSymbol(g_dtn_##tag, zn, sizeof(zn)) == cudaSuccess ? 0 : 1;        \
        }                                                                                         \
        return cudaMemcpyFromSymbol(host, g_dtr_##tag, sizeof(g_dtr_##tag)) == cudaSuccess ? 0 : 1; \
    }
#define DTRACE_START(tag, k)                                                                      \
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {                                 \
        unsigned long long t_;                                                                    \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
        const unsigned s_ = atomicAdd(&g_dtn_##tag[k], 1) & 63;                                    \
        g_dtc_##tag[k] = s_;                                                                      \
        g_dtr_##tag[k][s_][0] = t_;                                                               \
    }
#define DTRACE_WAITED(tag, k)                                                                     \
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {                                 \
        unsigned long long t_;                                                                    \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
        g_dtr_##tag[k][g_dtc_##tag[k]][1] = t_;                                                   \
    }
#define DTRACE_MARK(tag, k, f)                                                                    \
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {                                 \
        unsigned long long t_;                                                                    \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
        g_dtr_##tag[k][g_dtc_##tag[k]][f] = t_;                                                   \
    }
#define DTRACE_END(tag, k)                                                                        \
    if (threadIdx.x == 0) {                                                                       \
        unsigned long long t_;                                                                    \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
        atomicMax(&g_dtr_##tag[k][*(volatile unsigned *)&g_dtc_##tag[k]][2], t_);                 \
    }
#else
#define DTRACE_DEFINE(tag)
#define DTRACE_START(tag, k)
#define DTRACE_WAITED(tag, k)
#define DTRACE_MARK(tag, k, f)
#define DTRACE_END(tag, k)
#endif

__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes, int tid, int nthreads) {
    const char *c = static_cast<const char *>(p);
    for (size_t o = (size_t)tid * 128; o < bytes; o += (size_t)nthreads * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
}
}  // namespace ofb
