// dequant.cu — Q4_K / Q6_K super-block decode on the device, bit-identical to
// the reference's CPU decode (engine/src/gguf.c:43-86 whole-tensor,
// :511-571 single element, :605-711 public entry points).
//
// HBM-bound: a Q4_K block is 144 B in / 1024 B out (f32), a Q6_K block
// 210 B in / 1024 B out. One warp decodes one block (Q4_K) or a run of 8
// blocks staged through shared memory (Q6_K, whose 210-byte blocks are only
// 2-byte aligned; 8 blocks = 1680 B = 105 aligned 16-byte words). Each lane
// writes 8 consecutive outputs, so a warp stores one contiguous 1 KB row.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace ofb {

template <typename OutT>
__device__ __forceinline__ void store8(OutT *dst, const float v[8]);

template <>
__device__ __forceinline__ void store8<float>(float *dst, const float v[8]) {
    reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16 *dst, const float v[8]) {
    uint4 w;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]);
    __nv_bfloat162 p3 = __floats2bfloat162_rn(v[6], v[7]);
    w.x = *reinterpret_cast<uint32_t *>(&p0);
    w.y = *reinterpret_cast<uint32_t *>(&p1);
    w.z = *reinterpret_cast<uint32_t *>(&p2);
    w.w = *reinterpret_cast<uint32_t *>(&p3);
    *reinterpret_cast<uint4 *>(dst) = w;
}

template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Lane L of the warp owns the 8 outputs [8L, 8L+8) of the block: chunk
// c = L/8 (32 qs bytes, 64 outputs), low nibbles for L%8 < 4, else high.
template <typename OutT>
__global__ void __launch_bounds__(256) q4k_dequant_kernel(const uint8_t *__restrict__ blocks,
                                                          uint64_t n_blocks,
                                                          OutT *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    const uint64_t n_warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const int c = lane >> 3, k = lane & 7, hi = k >> 2, kk = k & 3;
    for (uint64_t b = warp; b < n_blocks; b += n_warps) {
        const uint8_t *blk = blocks + b * Q4K_BYTES;
        uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
        uint2 q = __ldg(reinterpret_cast<const uint2 *>(blk + 16 + c * 32 + kk * 8));
        float d = half_bits_ref(hdr.x & 0xFFFFu);
        float dmin = half_bits_ref(hdr.x >> 16);
        uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
        int sc, mn;
        q4k_scale_min(s, 2 * c + hi, sc, mn);
        float dsc = __fmul_rn(d, (float)sc);
        float dmm = __fmul_rn(dmin, (float)mn);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t byte = ((i < 4 ? q.x : q.y) >> (8 * (i & 3))) & 0xFFu;
            int qv = hi ? (int)(byte >> 4) : (int)(byte & 0xF);
            v[i] = q4k_value(dsc, dmm, qv);
        }
        store8<OutT>(out + b * QK + lane * 8, v);
    }
}

// Decode of one Q6_K block held in shared memory; lane L owns outputs
// [8L, 8L+8): half = L/16, quad = (L/4)%4, l = 8*(L%4) + i.
template <typename OutT>
__device__ __forceinline__ void q6k_decode_lane(const uint8_t *blk, int lane, OutT *dst) {
    const int half = lane >> 4, quad = (lane >> 2) & 3, l0 = (lane & 3) * 8;
    const uint8_t *ql = blk + half * 64 + (quad & 1) * 32 + l0;
    const uint8_t *qh = blk + 128 + half * 32 + l0;
    int sc = (int)(int8_t)blk[192 + half * 8 + quad * 2 + (l0 >> 4)];
    float d = half_bits_ref((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
    float ds = __fmul_rn(d, (float)sc);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int nib = (quad < 2) ? (ql[i] & 0xF) : (ql[i] >> 4);
        int top = (qh[i] >> (2 * quad)) & 3;
        int qv = (nib | (top << 4)) - 32;
        v[i] = __fmul_rn(ds, (float)qv);
    }
    store8<OutT>(dst, v);
}

template <typename OutT>
__global__ void __launch_bounds__(256) q6k_dequant_kernel(const uint8_t *__restrict__ blocks,
                                                          uint64_t n_blocks,
                                                          OutT *__restrict__ out) {
    __shared__ __align__(16) uint8_t stage[8][8 * Q6K_BYTES];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    const uint64_t n_warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint64_t n_groups = (n_blocks + 7) / 8;
    uint8_t *st = stage[wib];
    for (uint64_t g = warp; g < n_groups; g += n_warps) {
        const uint64_t b0 = g * 8;
        const int nb = (int)((n_blocks - b0) < 8 ? (n_blocks - b0) : 8);
        const uint8_t *src = blocks + b0 * Q6K_BYTES;
        __syncwarp();
        if (nb == 8) {
            const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
            uint4 *d4 = reinterpret_cast<uint4 *>(st);
            for (int i = lane; i < 105; i += 32) d4[i] = __ldg(s4 + i);
        } else {
            const uint16_t *s2 = reinterpret_cast<const uint16_t *>(src);
            uint16_t *d2 = reinterpret_cast<uint16_t *>(st);
            for (int i = lane; i < nb * (Q6K_BYTES / 2); i += 32) d2[i] = __ldg(s2 + i);
        }
        __syncwarp();
        for (int j = 0; j < nb; j++)
            q6k_decode_lane<OutT>(st + j * Q6K_BYTES, lane, out + (b0 + j) * QK + lane * 8);
    }
}

template <typename OutT>
__global__ void f16_dequant_kernel(const uint16_t *__restrict__ src, uint64_t n,
                                   OutT *__restrict__ out) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = cvt_out<OutT>(half_bits_ref(src[i]));
}

template <typename OutT>
__global__ void f32_copy_kernel(const float *__restrict__ src, uint64_t n, OutT *__restrict__ out) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = cvt_out<OutT>(src[i]);
}

template <typename OutT>
__global__ void slice_kernel(const uint8_t *__restrict__ data, int type, uint64_t per_expert,
                             uint64_t n_experts, uint64_t expert, OutT *__restrict__ out) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < per_expert;
         i += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t lin = i * n_experts + expert;
        float v;
        if (type == OFB_TYPE_Q4_K)
            v = q4k_one(data + (lin / QK) * Q4K_BYTES, (int)(lin % QK));
        else if (type == OFB_TYPE_Q6_K)
            v = q6k_one(data + (lin / QK) * Q6K_BYTES, (int)(lin % QK));
        else if (type == OFB_TYPE_F16)
            v = half_bits_ref(reinterpret_cast<const uint16_t *>(data)[lin]);
        else
            v = reinterpret_cast<const float *>(data)[lin];
        out[i] = cvt_out<OutT>(v);
    }
}

template <typename OutT>
static int launch_dequant(const void *blocks, int type, uint64_t n_elems, OutT *out,
                          cudaStream_t s) {
    const int cap = sm_count() * 8;
    const uint8_t *b = static_cast<const uint8_t *>(blocks);
    if (type == OFB_TYPE_Q4_K) {
        uint64_t nb = n_elems / QK;
        if (nb) q4k_dequant_kernel<OutT><<<grid_for(nb, 8, cap), 256, 0, s>>>(b, nb, out);
    } else if (type == OFB_TYPE_Q6_K) {
        uint64_t nb = n_elems / QK;
        if (nb) q6k_dequant_kernel<OutT><<<grid_for((nb + 7) / 8, 8, cap), 256, 0, s>>>(b, nb, out);
    } else if (type == OFB_TYPE_F16) {
        if (n_elems)
            f16_dequant_kernel<OutT><<<grid_for(n_elems, 256, cap), 256, 0, s>>>(
                static_cast<const uint16_t *>(blocks), n_elems, out);
    } else {
        if (n_elems)
            f32_copy_kernel<OutT><<<grid_for(n_elems, 256, cap), 256, 0, s>>>(
                static_cast<const float *>(blocks), n_elems, out);
    }
    OFB_CHECK_LAUNCH("dequantize launch");
    return OFB_OK;
}

static bool type_ok(int t) {
    return t == OFB_TYPE_F32 || t == OFB_TYPE_F16 || t == OFB_TYPE_Q4_K || t == OFB_TYPE_Q6_K;
}

}  // namespace ofb

using namespace ofb;

extern "C" int ofb_dequantize(const void *blocks, int type, uint64_t n_elems, void *out,
                              int out_type, void *stream) {
    if (!blocks || !out) { set_error("ofb_dequantize: NULL pointer"); return OFB_EINVAL; }
    if (!type_ok(type)) { set_error("ofb_dequantize: unsupported type %d", type); return OFB_EINVAL; }
    if ((type == OFB_TYPE_Q4_K || type == OFB_TYPE_Q6_K) && (n_elems % QK)) {
        set_error("ofb_dequantize: n_elems %llu not a multiple of 256", (unsigned long long)n_elems);
        return OFB_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(blocks) & 15) || (reinterpret_cast<uintptr_t>(out) & 31)) {
        set_error("ofb_dequantize: blocks must be 16-byte and out 32-byte aligned");
        return OFB_EINVAL;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_type == OFB_OUT_F32) return launch_dequant<float>(blocks, type, n_elems, (float *)out, s);
    if (out_type == OFB_OUT_BF16)
        return launch_dequant<__nv_bfloat16>(blocks, type, n_elems, (__nv_bfloat16 *)out, s);
    set_error("ofb_dequantize: bad out_type %d", out_type);
    return OFB_EINVAL;
}

extern "C" int ofb_dequantize_expert_slice(const void *blocks, int type, uint64_t n_elems,
                                           uint64_t n_experts, int expert, void *out,
                                           int out_type, void *stream) {
    if (!blocks || !out) { set_error("expert_slice: NULL pointer"); return OFB_EINVAL; }
    if (expert < 0 || n_experts == 0 || (uint64_t)expert >= n_experts) {
        set_error("expert_slice: expert %d out of range [0,%llu)", expert, (unsigned long long)n_experts);
        return OFB_EINVAL;
    }
    if (!type_ok(type)) { set_error("expert_slice: unsupported type %d", type); return OFB_EINVAL; }
    if ((reinterpret_cast<uintptr_t>(blocks) & 15)) {
        set_error("expert_slice: blocks must be 16-byte aligned");
        return OFB_EINVAL;
    }
    uint64_t per = n_elems / n_experts;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int cap = sm_count() * 8;
    if (!per) return OFB_OK;
    if (out_type == OFB_OUT_F32)
        slice_kernel<float><<<grid_for(per, 256, cap), 256, 0, s>>>(
            (const uint8_t *)blocks, type, per, n_experts, (uint64_t)expert, (float *)out);
    else if (out_type == OFB_OUT_BF16)
        slice_kernel<__nv_bfloat16><<<grid_for(per, 256, cap), 256, 0, s>>>(
            (const uint8_t *)blocks, type, per, n_experts, (uint64_t)expert, (__nv_bfloat16 *)out);
    else { set_error("expert_slice: bad out_type %d", out_type); return OFB_EINVAL; }
    OFB_CHECK_LAUNCH("expert_slice launch");
    return OFB_OK;
}
