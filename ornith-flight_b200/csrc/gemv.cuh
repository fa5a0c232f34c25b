// gemv.cuh — device pieces of the dp4a dequant-GEMV kernels (decode-sized
// batches): SiLU as the reference rounds it, Q4_K row items against 16-bit
// quantised activations, 2-byte aligned shared-memory reads for Q6_K rows.
#pragma once
#include "common.cuh"

namespace ofb {

__device__ __forceinline__ float silu_ref_d(float g) {
    // engine/src/model.c:340-344
    if (g < -50.0f) return 0.0f;
    if (g > 50.0f) return g;
    return g / (1.0f + expf(-g));
}

__device__ __forceinline__ int dp4a_s(int a, int b, int c) { return __dp4a(a, b, c); }
__device__ __forceinline__ int dp4a_u(unsigned a, unsigned b, int c) {
    return (int)__dp4a(a, b, (unsigned)c);
}

__device__ __forceinline__ uint32_t comp(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One lane item of a Q4_K row: chunk c of a block (sub-blocks 2c and 2c+1,
// 32 quant bytes) against the quantised activations of the same 64 elements.
__device__ __forceinline__ float q4k_item_q(const uint4 &hdr, const uint4 &qa, const uint4 &qb, int c,
                                            const uint4 xh[4], const uint4 xl[4], float s_lo,
                                            float s_hi, float xs_lo, float xs_hi) {
    int ih_lo = 0, il_lo = 0, ih_hi = 0, il_hi = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t q = (w < 4) ? comp(qa, w) : comp(qb, w - 4);
        const uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;
        ih_lo = dp4a_s((int)lo, (int)comp(xh[w >> 2], w & 3), ih_lo);
        il_lo = dp4a_u(lo, comp(xl[w >> 2], w & 3), il_lo);
        ih_hi = dp4a_s((int)hi, (int)comp(xh[2 + (w >> 2)], w & 3), ih_hi);
        il_hi = dp4a_u(hi, comp(xl[2 + (w >> 2)], w & 3), il_hi);
    }
    const uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    int sc0, m0, sc1, m1;
    q4k_scale_min(s, 2 * c, sc0, m0);
    q4k_scale_min(s, 2 * c + 1, sc1, m1);
    const float d = half_bits_ref(hdr.x & 0xFFFFu), dmin = half_bits_ref(hdr.x >> 16);
    const float S_lo = (float)(ih_lo * 256 + il_lo), S_hi = (float)(ih_hi * 256 + il_hi);
    return d * ((float)sc0 * s_lo * S_lo + (float)sc1 * s_hi * S_hi) -
           dmin * ((float)m0 * xs_lo + (float)m1 * xs_hi);
}

// 4 bytes at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_u32_2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(b[0], b[1], (unsigned)(a & 3) * 8);
}

// Quantised h of one item (16 values: 4 quads x 4) of one token, as the
// dp4a loop consumes it: int8 high / uint8 low planes, the element sum, and
// the scale, per quad.
struct HQuad { uint32_t hh, hl; int xs; float sq; };


// Quantises the four h values of one (item, quad) cell (positions l0..l0+3
// of a 16-element Q6_K scale group); the four lanes of a scale group are
// adjacent lanes of the warp, and every lane of the warp must call this.
__device__ __forceinline__ HQuad quantize_hquad(float4 hv) {
    float m = fmaxf(fmaxf(fabsf(hv.x), fabsf(hv.y)), fmaxf(fabsf(hv.z), fabsf(hv.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float sc = m / 32767.0f;
    const float inv = (m > 0.f) ? 32767.0f / m : 0.f;
    const int i0 = __float2int_rn(hv.x * inv), i1 = __float2int_rn(hv.y * inv);
    const int i2 = __float2int_rn(hv.z * inv), i3 = __float2int_rn(hv.w * inv);
    HQuad q;
    q.hh = ((uint32_t)(i0 >> 8) & 0xFF) | (((uint32_t)(i1 >> 8) & 0xFF) << 8) |
           (((uint32_t)(i2 >> 8) & 0xFF) << 16) | (((uint32_t)(i3 >> 8) & 0xFF) << 24);
    q.hl = (uint32_t)(i0 & 255) | ((uint32_t)(i1 & 255) << 8) | ((uint32_t)(i2 & 255) << 16) |
           ((uint32_t)(i3 & 255) << 24);
    q.xs = i0 + i1 + i2 + i3;
    q.sq = sc;
    return q;
}

// One lane item j of a Q6_K row in shared memory (2-byte aligned): the 16
// weights at positions l0..l0+3 of the four quads of half `half` of block b,
// against the quantised h of the same positions (hp[0..3], one per quad).
// Returns d * sum over the quads of scale * (h . q).
__device__ __forceinline__ float q6k_item_q(const uint8_t *row, int j, const HQuad *hp) {
    const int b = j >> 4, half = (j >> 3) & 1, l0 = (j & 7) * 4;
    const uint8_t *blk = row + b * Q6K_BYTES;
    const uint32_t W1 = lds_u32_2(blk + half * 64 + l0);
    const uint32_t W2 = lds_u32_2(blk + half * 64 + 32 + l0);
    const uint32_t Qh = lds_u32_2(blk + 128 + half * 32 + l0);
    const uint32_t SC0 = lds_u32_2(blk + 192 + half * 8);
    const uint32_t SC1 = lds_u32_2(blk + 192 + half * 8 + 4);
    const uint32_t DW = lds_u32_2(blk + 208);
    const uint32_t qv[4] = {(W1 & 0x0F0F0F0Fu) | ((Qh << 4) & 0x30303030u),
                            (W2 & 0x0F0F0F0Fu) | ((Qh << 2) & 0x30303030u),
                            ((W1 >> 4) & 0x0F0F0F0Fu) | (Qh & 0x30303030u),
                            ((W2 >> 4) & 0x0F0F0F0Fu) | ((Qh >> 2) & 0x30303030u)};
    const int is = l0 >> 4;
    float acc = 0.f;
#pragma unroll
    for (int quad = 0; quad < 4; quad++) {
        const uint4 v = *reinterpret_cast<const uint4 *>(hp + quad);
        const int sidx = quad * 2 + is;  // scales[half*8 + 2*quad + is]
        const uint32_t scw = sidx < 4 ? SC0 : SC1;
        const int scale = (int)(int8_t)(scw >> (8 * (sidx & 3)));
        const int S = dp4a_s((int)qv[quad], (int)v.x, 0) * 256 + dp4a_u(qv[quad], v.y, 0) - 32 * (int)v.z;
        acc += (float)scale * __uint_as_float(v.w) * (float)S;
    }
    return half_bits_ref(DW & 0xFFFFu) * acc;
}

}  // namespace ofb
