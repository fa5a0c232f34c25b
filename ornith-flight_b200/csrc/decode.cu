// decode.cu — expert kernels for decode-sized batches (T <= 32 tokens).
//
// HBM-bound: at batch 1 a layer reads ~20 MB of Q4_K/Q6_K weights once, so
// the kernels are built to keep many 16-byte loads in flight and to spend
// about one instruction per weight:
//  * activations are pre-quantised per 32 (x) or 16 (h) elements to a 16-bit
//    integer split into an int8 high plane and a uint8 low plane
//    (v ~= s * (256*hi + lo), |error| <= max|v|/65534 per element), so a
//    sub-block dot product is two dp4a chains on the raw 4-bit / 6-bit quants
//    followed by the block's own scale arithmetic. Relative error of a row
//    dot product is ~1e-5, well inside the layer's 1e-3 bound.
//  * expert_up_q: one warp per (slot, 2 hidden rows) streams the Q4_K gate
//    and up rows (lane = one 64-element chunk: 16 B header + 32 B quants),
//    writes h = silu(x.G) * (x.U) per token. It raises its dependent-launch
//    trigger once routing is known, so expert_down_q stages its rows while
//    this kernel runs.
//  * expert_down_q: one CTA per (slot, 64 output rows) stages the 64 Q6_K
//    rows (26,880 B, 16-byte aligned) in shared memory and quantises each
//    token's h once per CTA; warp w computes rows 4w..4w+3 and writes y per
//    assignment; the last warp to finish a group of 4 rows (atomic ticket)
//    adds resid + gate*shared + sum_a w_a*y_a in the reference's order
//    (model.c:1007, :1090, :1142), so the combine is deterministic and
//    needs no extra launch.
#include "common.cuh"
#include "moe.cuh"
#include "gemv.cuh"

namespace ofb {

DTRACE_DEFINE(dc)

__device__ __forceinline__ int asg_token_d(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

constexpr int UP_R = 2;  // hidden rows per warp

__global__ void __launch_bounds__(256) expert_up_q(LayerArgs a, const unsigned char *__restrict__ xq) {
    DTRACE_START(dc, 0)
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int D = a.D, nbr = D / QK, items = nbr * 4, TK = a.T * a.K;
    const size_t row_bytes = (size_t)nbr * Q4K_BYTES, exp_bytes = row_bytes * a.H;
    // the shared expert does not depend on routing: start pulling it into L2
    if (a.has_shared) {
        const int gt = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
        prefetch_l2(a.gate_sh, exp_bytes, gt, nt);
        prefetch_l2(a.up_sh, exp_bytes, gt, nt);
    }
    pdl_wait();
    // routing is complete: let expert_down_q start (it stages its Q6_K rows
    // from the plan while this kernel runs)
    pdl_trigger();
    DTRACE_WAITED(dc, 0)
    const size_t xs = xq_stride(D);
    const int groups = a.H / UP_R;
    const int units = *a.n_slots * groups;
    for (int unit = warp; unit < units; unit += nwarps) {
        const int u = unit / groups, m0 = (unit - u * groups) * UP_R;
        const int e = a.slot_expert[u];
        const uint8_t *G = (e == a.E ? a.gate_sh : a.gate + e * exp_bytes) + m0 * row_bytes;
        const uint8_t *U = (e == a.E ? a.up_sh : a.up + e * exp_bytes) + m0 * row_bytes;
        const int s1 = a.slot_start[u + 1];
        for (int s = a.slot_start[u]; s < s1; s++) {
            const int asg = a.assign[s];
            const unsigned char *q = xq + (size_t)asg_token_d(asg, TK, a.K) * xs;
            const float *qf = reinterpret_cast<const float *>(q + 2 * D);
            float ag[UP_R], au[UP_R];
#pragma unroll
            for (int r = 0; r < UP_R; r++) ag[r] = au[r] = 0.f;
            for (int j = lane; j < items; j += 32) {
                const int b = j >> 2, c = j & 3;
                uint4 hg[UP_R], ga[UP_R], gb[UP_R], hu[UP_R], ua[UP_R], ub[UP_R];
#pragma unroll
                for (int r = 0; r < UP_R; r++) {
                    const uint8_t *gblk = G + r * row_bytes + b * Q4K_BYTES;
                    const uint8_t *ublk = U + r * row_bytes + b * Q4K_BYTES;
                    hg[r] = __ldg(reinterpret_cast<const uint4 *>(gblk));
                    ga[r] = __ldg(reinterpret_cast<const uint4 *>(gblk + 16 + c * 32));
                    gb[r] = __ldg(reinterpret_cast<const uint4 *>(gblk + 32 + c * 32));
                    hu[r] = __ldg(reinterpret_cast<const uint4 *>(ublk));
                    ua[r] = __ldg(reinterpret_cast<const uint4 *>(ublk + 16 + c * 32));
                    ub[r] = __ldg(reinterpret_cast<const uint4 *>(ublk + 32 + c * 32));
                }
                const int e0 = b * QK + c * 64, sb = e0 / 32;
                uint4 xh[4], xl[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    xh[i] = __ldg(reinterpret_cast<const uint4 *>(q + e0) + i);
                    xl[i] = __ldg(reinterpret_cast<const uint4 *>(q + D + e0) + i);
                }
                const float s_lo = qf[sb], s_hi = qf[sb + 1];
                const float xs_lo = qf[D / 32 + sb], xs_hi = qf[D / 32 + sb + 1];
#pragma unroll
                for (int r = 0; r < UP_R; r++) {
                    ag[r] += q4k_item_q(hg[r], ga[r], gb[r], c, xh, xl, s_lo, s_hi, xs_lo, xs_hi);
                    au[r] += q4k_item_q(hu[r], ua[r], ub[r], c, xh, xl, s_lo, s_hi, xs_lo, xs_hi);
                }
            }
#pragma unroll
            for (int r = 0; r < UP_R; r++) {
                const float g = warp_sum(ag[r]), uu = warp_sum(au[r]);
                if (lane == 0) a.h[(size_t)asg * a.H + m0 + r] = silu_ref_d(g) * uu;
            }
        }
    }
    DTRACE_END(dc, 0)
}

// ---- down ------------------------------------------------------------------

constexpr int DG = DOWN_TICKET_ROWS;  // output rows per warp (one ticket each)
constexpr int DQ_WARPS = 16;  // warps per CTA
constexpr int DQ_ROWS = DG * DQ_WARPS;  // output rows per CTA
constexpr int DQ_TOK = 8;     // tokens whose quantised h is staged at once

// One CTA per (slot, 64 output rows): stage the 64 Q6_K rows in shared memory
// (the first unit's before waiting for expert_up_q, which runs meanwhile),
// quantise each token's h once per CTA (per 16-element Q6_K scale group),
// then warp w computes rows 4w..4w+3 for every token of the slot.
__global__ void __launch_bounds__(DQ_WARPS * 32) expert_down_q(LayerArgs a, int *__restrict__ tickets) {
    extern __shared__ __align__(16) uint8_t dsm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5, tid = threadIdx.x;
    const int D = a.D, H = a.H, nbk = H / QK, items = nbk * 16, TK = a.T * a.K;
    const int row_bytes = nbk * Q6K_BYTES;
    const size_t exp_bytes = (size_t)row_bytes * D;
    const int nblk = D / DQ_ROWS;
    DTRACE_START(dc, 1)
    pdl_trigger();
    if (a.has_shared) {
        const int gt = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
        prefetch_l2(a.down_sh, exp_bytes, gt, nt);
    }
    uint8_t *slab = dsm;                                                        // [64][row_bytes]
    HQuad *hq = reinterpret_cast<HQuad *>(dsm + DQ_ROWS * row_bytes + 16);     // [DQ_TOK][items][4]
    // The routing plan is complete when this grid starts: expert_up_q raises
    // its trigger only after its own wait on the routing kernel. So the first
    // unit's Q6_K rows are staged before waiting for h (plan read through L2).
    const int nslots = __ldcg(a.n_slots);
    const int units = nslots * nblk;
    auto stage_slab = [&](int unit) {
        const int u = unit / nblk, n0 = (unit - u * nblk) * DQ_ROWS;
        const int e = __ldcg(a.slot_expert + u);
        const uint8_t *src = (e == a.E ? a.down_sh : a.down + e * exp_bytes) + (size_t)n0 * row_bytes;
        for (int i = tid; i < DQ_ROWS * row_bytes / 16; i += DQ_WARPS * 32)
            reinterpret_cast<uint4 *>(slab)[i] = __ldg(reinterpret_cast<const uint4 *>(src) + i);
    };
    if ((int)blockIdx.x < units) stage_slab(blockIdx.x);
    pdl_wait();
    DTRACE_WAITED(dc, 1)
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
        const int u = unit / nblk, n0 = (unit - u * nblk) * DQ_ROWS;
        if (unit != (int)blockIdx.x) {
            __syncthreads();  // previous unit done with the slab and hq
            stage_slab(unit);
        }
        const int s0 = a.slot_start[u], s1 = a.slot_start[u + 1];
        DTRACE_MARK(dc, 1, 3)
        for (int c0 = s0; c0 < s1; c0 += DQ_TOK) {
            const int nc = min(DQ_TOK, s1 - c0);
            if (c0 > s0) __syncthreads();  // previous chunk's hq consumed
            // quantise h: thread p = (token, quad, item); the 4 items of a
            // scale group are adjacent lanes
            for (int p = tid; p < nc * 4 * items; p += DQ_WARPS * 32) {
                const int tk = p / (4 * items), rem = p - tk * 4 * items, quad = rem / items, j = rem - quad * items;
                const float *hrow = a.h + (size_t)a.assign[c0 + tk] * H;
                const int b = j >> 4, half = (j >> 3) & 1, l0 = (j & 7) * 4;
                const float4 hv = *reinterpret_cast<const float4 *>(hrow + b * QK + half * 128 + l0 + quad * 32);
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
                hq[(tk * items + j) * 4 + quad] = q;
            }
            __syncthreads();
            DTRACE_MARK(dc, 1, 4)
            for (int tk = 0; tk < nc; tk++) {
                const int asg = a.assign[c0 + tk];
                float yp[DG];
#pragma unroll
                for (int r = 0; r < DG; r++) yp[r] = 0.f;
                for (int j = lane; j < items; j += 32) {
                    const int b = j >> 4, half = (j >> 3) & 1, l0 = (j & 7) * 4;
                    const HQuad *hp = hq + (tk * items + j) * 4;
                    uint32_t HH[4], HL[4];
                    int XS[4];
                    float sq[4];
#pragma unroll
                    for (int quad = 0; quad < 4; quad++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(hp + quad);
                        HH[quad] = v.x;
                        HL[quad] = v.y;
                        XS[quad] = (int)v.z;
                        sq[quad] = __uint_as_float(v.w);
                    }
#pragma unroll
                    for (int r = 0; r < DG; r++) {
                        const uint8_t *blk = slab + (wib * DG + r) * row_bytes + b * Q6K_BYTES;
                        const uint32_t W1 = lds_u32_2(blk + half * 64 + l0);
                        const uint32_t W2 = lds_u32_2(blk + half * 64 + 32 + l0);
                        const uint32_t Qh = lds_u32_2(blk + 128 + half * 32 + l0);
                        const uint32_t SC0 = lds_u32_2(blk + 192 + half * 8);
                        const uint32_t SC1 = lds_u32_2(blk + 192 + half * 8 + 4);
                        const uint32_t DW = lds_u32_2(blk + 208);
                        const uint32_t qv[4] = {
                            (W1 & 0x0F0F0F0Fu) | ((Qh << 4) & 0x30303030u),
                            (W2 & 0x0F0F0F0Fu) | ((Qh << 2) & 0x30303030u),
                            ((W1 >> 4) & 0x0F0F0F0Fu) | (Qh & 0x30303030u),
                            ((W2 >> 4) & 0x0F0F0F0Fu) | ((Qh >> 2) & 0x30303030u)};
                        const int is = l0 >> 4;
                        float acc = 0.f;
#pragma unroll
                        for (int quad = 0; quad < 4; quad++) {
                            const int sidx = quad * 2 + is;  // scales[half*8 + 2*quad + is]
                            const uint32_t scw = sidx < 4 ? SC0 : SC1;
                            const int scale = (int)(int8_t)(scw >> (8 * (sidx & 3)));
                            const int S = dp4a_s((int)qv[quad], (int)HH[quad], 0) * 256 +
                                          dp4a_u(qv[quad], HL[quad], 0) - 32 * XS[quad];
                            acc += (float)scale * sq[quad] * (float)S;
                        }
                        yp[r] += half_bits_ref(DW & 0xFFFFu) * acc;
                    }
                }
#pragma unroll
                for (int r = 0; r < DG; r++) {
                    const float v = warp_sum(yp[r]);
                    if (lane == 0) a.y[(size_t)asg * D + n0 + wib * DG + r] = v;
                }
            }
        }
        DTRACE_MARK(dc, 1, 5)
        // the last slot to finish a group of 4 rows combines them
        const int g = n0 / DG + wib;
        int last = 0;
        if (lane == 0) {
            __threadfence();
            last = (atomicAdd(&tickets[g], 1) == nslots - 1);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            const int m0 = n0 + wib * DG;
            for (int p = lane; p < a.T * DG; p += 32) {
                const int t = p / DG, n = m0 + (p - t * DG);
                const size_t o = (size_t)t * D + n;
                float acc = a.resid ? a.resid[o] : 0.f;
                if (a.has_shared) {
                    const float ys = __ldcg(a.y + (size_t)(TK + t) * D + n);
                    acc += a.shared_gate ? a.gsc[t] * ys : ys;
                }
                float rr = 0.f;
                for (int k = 0; k < a.K; k++) {
                    const int asg = t * a.K + k;
                    const float w = __ldcg(a.w + asg);
                    if (w < 1e-6f) continue;
                    rr += w * __ldcg(a.y + (size_t)asg * D + n);
                }
                a.out[o] = acc + rr;
            }
            if (lane == 0) tickets[g] = 0;
        }
    }
    DTRACE_END(dc, 1)
}

__global__ void quantize_x_kernel(const float *__restrict__ x, int D, unsigned char *__restrict__ xq) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.y;
    const float *xt = x + (size_t)t * D;
    unsigned char *q = xq + (size_t)t * xq_stride(D);
    for (int sb = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); sb < D / 32;
         sb += gridDim.x * (blockDim.x >> 5)) {
        const float v = xt[sb * 32 + lane];
        float m = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float s = m / 32767.0f;
        const int xi = (m > 0.0f) ? __float2int_rn(v / s) : 0;
        q[sb * 32 + lane] = (unsigned char)(xi >> 8);
        q[D + sb * 32 + lane] = (unsigned char)(xi & 255);
        const float xsum = warp_sum(v);
        if (lane == 0) {
            reinterpret_cast<float *>(q + 2 * D)[sb] = s;
            reinterpret_cast<float *>(q + 2 * D)[D / 32 + sb] = xsum;
        }
    }
}

int launch_quantize_x(const float *x, int T, int D, unsigned char *xq, cudaStream_t s) {
    dim3 grid((D / 32 + 7) / 8, T);
    quantize_x_kernel<<<grid, 256, 0, s>>>(x, D, xq);
    OFB_CHECK_LAUNCH("quantize_x");
    return OFB_OK;
}

int launch_up_q(const LayerArgs &a, const unsigned char *xq, int max_slots, cudaStream_t s) {
    const uint64_t up_units = (uint64_t)max_slots * (a.H / UP_R);
    cudaError_t e = launch_pdl(expert_up_q, dim3(grid_for(up_units, 8, sm_count() * 32)), dim3(256), 0, s, a, xq);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "expert_up_q launch");
}

int launch_down_q(const LayerArgs &a, int *tickets, int max_slots, cudaStream_t s) {
    const int n = sm_count();
    const size_t smem = (size_t)DQ_ROWS * (a.H / QK) * Q6K_BYTES + 16 + (size_t)DQ_TOK * (a.H / QK) * 16 * 4 * sizeof(HQuad);
    static size_t attr[64];
    cudaError_t ea = ensure_dyn_smem(expert_down_q, smem, attr);
    if (ea != cudaSuccess) return cuda_status(ea, "expert_down_q smem attribute");
    const uint64_t dn_units = (uint64_t)max_slots * (a.D / DQ_ROWS);
    const int grid = (int)(dn_units < (uint64_t)n * 4 ? dn_units : (uint64_t)n * 4);
    cudaError_t e = launch_pdl(expert_down_q, dim3(grid), dim3(DQ_WARPS * 32), smem, s, a, tickets);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "expert_down_q launch");
}

}  // namespace ofb
