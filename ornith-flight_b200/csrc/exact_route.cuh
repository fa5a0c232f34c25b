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

__device__ __forceinline__ void xl_cp16(float *dst, const float *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// Reference-order logit of one router row by one lane of a warp, the row
// streamed through this lane's ST chunk slots of XL_CK floats (cp.async,
// ST - 1 chunks in flight). `slots` = this lane's first slot; slot c of lane
// l sits at (c * 32 + l) * XL_LD floats from the warp's base, so a warp's
// 16-byte reads of one chunk position fall in distinct banks. D % XL_CK == 0.
// Only this lane's copies are waited for: no barrier, so the chain (2048
// dependent adds at d_model 2048) is the only floor.
constexpr int XL_CK = 64, XL_LD = XL_CK + 4;
template <int ST>
__device__ float exact_logit_lane(const float *__restrict__ wrow, const float *xs, int D, float *slots) {
    const int nch = D / XL_CK;
    auto issue = [&](int ch) {
        if (ch < nch) {
            float *dst = slots + (ch % ST) * 32 * XL_LD;
#pragma unroll
            for (int q = 0; q < XL_CK / 4; q++) xl_cp16(dst + 4 * q, wrow + ch * XL_CK + 4 * q);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int c = 0; c < ST - 1; c++) issue(c);
    float s = 0.0f;
    for (int ch = 0; ch < nch; ch++) {
        issue(ch + ST - 1);  // its slot was read by chunk ch - 1
        asm volatile("cp.async.wait_group %0;" ::"n"(ST - 1) : "memory");
        const float *wc = slots + (ch % ST) * 32 * XL_LD, *xc = xs + ch * XL_CK;
#pragma unroll
        for (int k = 0; k < XL_CK; k += 4) {
            const float4 w4 = *reinterpret_cast<const float4 *>(wc + k);
            const float4 x4 = *reinterpret_cast<const float4 *>(xc + k);
            s = __fadd_rn(s, __fmul_rn(x4.x, w4.x));
            s = __fadd_rn(s, __fmul_rn(x4.y, w4.y));
            s = __fadd_rn(s, __fmul_rn(x4.z, w4.z));
            s = __fadd_rn(s, __fmul_rn(x4.w, w4.w));
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    return s;
}

// The same chains for a list of experts: warp 0 of the calling block runs
// them, lane c on expert list[c] (32 at a time), each lane streaming its own
// router row (exact_logit_lane); the other threads return at once. The
// caller synchronises the block before reading out[c] = logit of list[c].
// wbuf: XL_SMEM bytes of shared memory, 16-byte aligned.
constexpr int XL_ST = 7;                               // chunk slots per lane
constexpr int XL_SMEM = XL_ST * 32 * XL_LD * 4;        // 60,928 bytes
static __device__ void exact_logits_block(const float *__restrict__ W, int D, const float *xs, const int *list, int n,
                                          float *out, float *wbuf, int tid, int nthreads) {
    (void)nthreads;
    if (tid >= 32) return;
    for (int c = tid; c < n; c += 32) out[c] = exact_logit_lane<XL_ST>(W + (size_t)list[c] * D, xs, D, wbuf + tid * XL_LD);
}

__device__ __forceinline__ bool close_ulps(float a, float b, int ulps) {
    int ia = __float_as_int(a), ib = __float_as_int(b);  // non-negative floats
    return abs(ia - ib) <= ulps;
}

}  // namespace ofb
