// exact_route.cuh — the reference's router logit chain (sequential fp32,
// product then add, engine/src/model.c:1019-1025), per thread and for a list
// of experts computed by a whole block; used where the certified routing
// cannot decide the top-k from bounded approximations.
#pragma once
#include "common.cuh"

namespace ofb {

// Reference-order logit: sequential fp32, product then add, d = 0..D-1.
// The router row streams through registers in 64-element chunks, the next
// chunk loading while the chain runs over the current one (the 2048-step
// add chain is the latency floor).
static __device__ float exact_logit(const float *wrow, const float *xs, int D) {
    constexpr int C = 16;  // float4 per chunk
    const float4 *w4 = reinterpret_cast<const float4 *>(wrow);
    float4 cur[C], nxt[C];
#pragma unroll
    for (int j = 0; j < C; j++) cur[j] = __ldg(w4 + j);
    float s = 0.0f;
    for (int c0 = 0; c0 < D / 4; c0 += C) {
        if (c0 + C < D / 4) {
#pragma unroll
            for (int j = 0; j < C; j++) nxt[j] = __ldg(w4 + c0 + C + j);
        }
#pragma unroll
        for (int j = 0; j < C; j++) {
            const float4 x4 = *reinterpret_cast<const float4 *>(xs + 4 * (c0 + j));
            s = __fadd_rn(s, __fmul_rn(x4.x, cur[j].x));
            s = __fadd_rn(s, __fmul_rn(x4.y, cur[j].y));
            s = __fadd_rn(s, __fmul_rn(x4.z, cur[j].z));
            s = __fadd_rn(s, __fmul_rn(x4.w, cur[j].w));
        }
#pragma unroll
        for (int j = 0; j < C; j++) cur[j] = nxt[j];
    }
    return s;
}

// The same chains for a list of experts, computed by the whole block: the
// threads stage 256-element chunks of up to 32 router rows in shared memory
// (cp.async, two buffers, rows padded by 4 floats so the chain threads' float4
// reads are conflict-free) and thread c < 32 runs expert list[c]'s chain
// over each chunk. Every thread of the block calls this; out[c] = logit of
// list[c].
constexpr int XL_CK = 256, XL_LD = XL_CK + 4, XL_ROWS = 32;
constexpr int XL_SMEM = 2 * XL_ROWS * XL_LD * 4;  // bytes of the two chunk buffers

__device__ __forceinline__ void xl_cp16(float *dst, const float *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

static __device__ void exact_logits_block(const float *__restrict__ W, int D, const float *xs, const int *list, int n,
                                   float *out, float *wbuf, int tid, int nthreads) {
    const int nch = (D + XL_CK - 1) / XL_CK;
    for (int g0 = 0; g0 < n; g0 += XL_ROWS) {
        const int ng = min(XL_ROWS, n - g0);
        auto issue = [&](int ch) {
            float *dst = wbuf + (ch & 1) * XL_ROWS * XL_LD;
            const int k0 = ch * XL_CK, q4 = min(XL_CK, D - k0) / 4;
            for (int i = tid; i < ng * q4; i += nthreads) {
                const int r = i / q4, q = i - r * q4;
                xl_cp16(dst + r * XL_LD + 4 * q, W + (size_t)list[g0 + r] * D + k0 + 4 * q);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        float s = 0.0f;
        issue(0);
        for (int ch = 0; ch < nch; ch++) {
            if (ch + 1 < nch) {
                issue(ch + 1);
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncthreads();
            if (tid < ng) {
                const float *wr = wbuf + (ch & 1) * XL_ROWS * XL_LD + tid * XL_LD;
                const float *xc = xs + ch * XL_CK;
                const int cw = min(XL_CK, D - ch * XL_CK);
#pragma unroll 8
                for (int k = 0; k < cw; k += 4) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(wr + k);
                    const float4 x4 = *reinterpret_cast<const float4 *>(xc + k);
                    s = __fadd_rn(s, __fmul_rn(x4.x, w4.x));
                    s = __fadd_rn(s, __fmul_rn(x4.y, w4.y));
                    s = __fadd_rn(s, __fmul_rn(x4.z, w4.z));
                    s = __fadd_rn(s, __fmul_rn(x4.w, w4.w));
                }
            }
            __syncthreads();  // the buffer is refilled next chunk
        }
        if (tid < ng) out[g0 + tid] = s;
    }
}

__device__ __forceinline__ bool close_ulps(float a, float b, int ulps) {
    int ia = __float_as_int(a), ib = __float_as_int(b);  // non-negative floats
    return abs(ia - ib) <= ulps;
}

}  // namespace ofb
