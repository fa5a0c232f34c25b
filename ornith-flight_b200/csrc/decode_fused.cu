// decode_fused.cu — the whole MoE layer for one token (decode batch 1) in a
// single persistent launch: router, softmax/top-k/renormalise, expert SwiGLU
// on the raw Q4_K/Q6_K blocks, sigmoid-gated shared expert and the combine
// (engine/src/model.c:992-1143 for one token).
//
// Why one launch: at batch 1 the layer moves ~20 MB (3.1 us of HBM time)
// through four dependent steps (router -> top-k -> gate/up -> down). As
// separate kernels each step pays a launch hand-off and a ramp of its own;
// here every CTA moves its share of every step's bytes with bulk copies
// (TMA, cp.async.bulk) into shared memory as soon as it knows the addresses,
// and CTAs exchange the few values that cross between steps: router logits
// with bounds (tagged 64-bit words) and the quantised h of each expert (one
// global image, brought into every CTA by one bulk copy).
//
// One CTA per SM (grid = SM count, ~190 KB of shared memory each). In units
// of 16-row h groups (fd_share), CTA c owns
//  * router rows c, c+G, ... (and the shared-expert gate vector as row E),
//  * routed (slot, hidden row) pairs [u0, u1) in top-k slot order, and, on
//    the CTAs with the fewest of those, shared-expert hidden rows [s0, s1),
//  * output rows [n0, n1) (groups of dg rows, 16-byte aligned Q6_K slabs),
//    for every expert: the CTA computes y of all K+1 experts for its rows and
//    combines them in the reference's order, so no cross-CTA reduction.
// Steps:
//  0. before the dependent-launch wait (the previous kernel may still run):
//     bulk copies of the static bytes it owns: router rows, shared gate/up
//     rows, shared down rows.
//  1. x (bulk copy) -> 16-bit quantised copy for dp4a; router logits of its
//     rows as float pairs with a rigorous bound B of the distance to the
//     reference's sequential fp32 sum (the certified routing of
//     route_fast.cu, restated per CTA), published as tagged words.
//  2. every CTA reads all (L~, B) and runs the same certified selection
//     (identical inputs, identical result): top-k indices bit-exact, or the
//     exact recompute of the uncertain candidates with the reference's chain
//     and the host C library's expf; then bulk copies of its routed gate/up
//     rows and of its output rows' Q6_K slabs of the K routed experts.
//     Meanwhile the other half of the warps quantise x and compute, quantise
//     and publish the CTA's shared-expert h groups.
//  3. routed h rows (dp4a on the raw nibbles); each 16-row group quantised
//     (per-group scale, int8 high / uint8 low planes) by the CTA that
//     computed it, stored into the global slot image and counted.
//  4. once every group is counted: one bulk copy of all slots; y for its
//     rows -> out = resid + g*y_sh + sum_k w_k y_k.
// Tags and counter targets come from the launch epoch + 1: a device counter
// advanced by the last CTA to finish publishing (every CTA has read the epoch
// by then), read after the dependent-launch wait
// (which orders it after the previous launch), so stale words from earlier
// launches never match and the kernel can be replayed (e.g. in a CUDA graph)
// without host bookkeeping. Every wait (mbarrier, tag, counter) is bounded; on
// expiry the CTA records an error bit in the workspace and runs to its exit on
// whatever it has.
//
// Requirements (checked on the host): T = 1, contiguous layout, router
// present, E <= 256 (selection by one warp), E + 1 <= 2 * grid, top_k <= 16,
// the per-CTA shares fit in shared memory.
#include <algorithm>

#include "async.cuh"
#include "common.cuh"
#include "exact_expf.h"
#include "exact_route.cuh"
#include "exchange.cuh"
#include "gemv.cuh"
#include "moe.cuh"

namespace ofb {

constexpr int FD_THREADS = 512;
constexpr int FD_WARPS = FD_THREADS / 32;
constexpr int FD_PER_LANE = 8;                            // selection: experts per lane (E <= 256)
constexpr unsigned long long FD_WAIT_NS = 500000000ull;  // 0.5 s per wait
constexpr int FD_GROUP_BYTES = 48;  // staging of one quantised h group (40 bytes used)
constexpr double FD_MARGIN = 0x1.0p-14;                   // certificate margin (as route_fast.cu)

// Error bits recorded in sync[2] (read by ofb_workspace_check).
constexpr uint32_t FD_ERR_COPY = 1u, FD_ERR_TAG = 2u;

struct FusedDecodeArgs {
    const float *W, *x, *gate_v, *resid;
    float *out;
    const uint8_t *gate, *up, *down, *gate_sh, *up_sh, *down_sh;
    int D, H, E, K, routing, renorm, has_shared, use_gate;
    double bound_scale, ngam;
    unsigned long long *cand;  // [2E + 1]: (L~, B) per expert, then the shared gate
    unsigned long long *hll;   // global image of the K + 1 quantised h slots (hslot layout)
    unsigned int *sync;        // [0] epoch, [1] CTAs finished, [2] error bits, [3] router rows
                               // published, [4 + k] h rows published of slot k (k <= K)
    uint32_t *idx_out;
    float *w_out;
    int *stats;  // [3] tokens per routing path (certified, candidates, full)
    FusedPlan p;
};

// Optional per-CTA timeline (build with -DOFB_FD_TRACE): globaltimer at each
// step boundary of the last launch, read back with ofb_debug_fd_trace.
#ifdef OFB_FD_TRACE
__device__ unsigned long long g_fd_tr[256][64];
#define FD_MARK_IF(cond, i) \
    if ((cond) && blockIdx.x < 256) g_fd_tr[blockIdx.x][i] = ax::gtime();
#else
#define FD_MARK_IF(cond, i)
#endif
#define FD_MARK(i) FD_MARK_IF(threadIdx.x == 0, i)

__device__ __forceinline__ float f_of(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t u_of(float f) { return __float_as_uint(f); }

// ---- gate/up rows on the tensor cores (mma.sync m16n8k32, u8 x s8 -> s32) ----
// A tile is 8 row pairs: rows 0-7 gate rows, rows 8-15 the same pairs' up
// rows; row g of a tile lies in shared-memory area g of its segment (see
// FdSegs), areas RS bytes apart with RS % 128 == 32, so the 4 rows a
// half-warp reads fall in different banks. One MMA covers one 32-weight
// Q4_K sub-block: A = its 4-bit quants (0..15), B = the activations as 16-bit
// integers x_int = 128 * hi + lo (hi int8, lo 0..127) of the same positions.
// Sub-block j puts hi / lo in B columns 2(j%4) / 2(j%4)+1 (other columns
// zero), so four consecutive sub-blocks accumulate into one C, and lane
// (g, tig) then holds the sums of sub-block 4m+tig for gate row g (c0, c1)
// and up row g (c2, c3). The k order inside a sub-block is permuted so that
// a lane's A and B registers are 8 consecutive bytes each: MMA k = 4 tig + i
// is byte 8 tig + i, k = 16 + 4 tig + i is byte 8 tig + 4 + i.
// Per sub-block j of a row: sum_i w_i x_i ~= s_j (d sc_j S - dmin m_j xsum_j)
// with S = sum_i q_i x_int,i = 128 c_hi + c_lo (exact in int32), s_j the
// activations' scale and xsum_j the sum of their (unquantised) values.
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(  // a pure function of its operands: free to schedule
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Partial (gate, up) dot products of tile t over Q4_K blocks [b0, b1) for
// pair 8t + g (returned on the lanes with tig == 0). G / U: the tile's first
// gate / up row; xq7: hi plane, lo plane (D bytes each), then per 32
// elements the scale s_j and xsum_j (floats).
__device__ __forceinline__ float2 tile_dots(const uint8_t *G, const uint8_t *U, int RS, int b0, int b1,
                                            const unsigned char *xq7, int D, int lane) {
    const int g = lane >> 2, tig = lane & 3;
    const uint8_t *gr = G + (size_t)g * RS, *ur = U + (size_t)g * RS;
    const float *xs = reinterpret_cast<const float *>(xq7 + 2 * D), *xsum = xs + D / 32;
    // B source of this lane: column n = g is plane (g & 1) of sub-block pair slot (g >> 1)
    const unsigned char *xpl = xq7 + (g & 1) * D + 8 * tig;
    float ag = 0.f, au = 0.f;
    for (int b = b0; b < b1; b++) {
        const uint4 hg = *reinterpret_cast<const uint4 *>(gr + b * Q4K_BYTES);
        const uint4 hu = *reinterpret_cast<const uint4 *>(ur + b * Q4K_BYTES);
        const float dg = half_bits_ref(hg.x & 0xFFFFu), dmg = half_bits_ref(hg.x >> 16);
        const float du = half_bits_ref(hu.x & 0xFFFFu), dmu = half_bits_ref(hu.x >> 16);
#pragma unroll
        for (int m = 0; m < 2; m++) {  // sub-blocks 4m .. 4m+3 of the block
            int cc[4] = {0, 0, 0, 0};
#pragma unroll
            for (int ch = 0; ch < 2; ch++) {  // 32-byte chunk 2m + ch: sub-blocks 2(2m+ch), 2(2m+ch)+1
                const int chunk = 2 * m + ch;
                const uint2 wg = *reinterpret_cast<const uint2 *>(gr + b * Q4K_BYTES + 16 + 32 * chunk + 8 * tig);
                const uint2 wu = *reinterpret_cast<const uint2 *>(ur + b * Q4K_BYTES + 16 + 32 * chunk + 8 * tig);
#pragma unroll
                for (int hi = 0; hi < 2; hi++) {
                    const int jj = 2 * ch + hi;  // sub-block within the group of four
                    const int j = b * 8 + 4 * m + jj;
                    uint2 bx = make_uint2(0u, 0u);
                    if ((g >> 1) == jj) bx = *reinterpret_cast<const uint2 *>(xpl + 32 * j);
                    const uint32_t sh = 4 * hi;
                    mma_u8s8(cc, (wg.x >> sh) & 0x0F0F0F0Fu, (wu.x >> sh) & 0x0F0F0F0Fu, (wg.y >> sh) & 0x0F0F0F0Fu,
                             (wu.y >> sh) & 0x0F0F0F0Fu, bx.x, bx.y);
                }
            }
            // epilogue: this lane's sub-block 4m + tig of the block
            const int jb = 4 * m + tig, j = b * 8 + jb;
            const float sx = xs[j], xm = xsum[j];
            {
                const uint32_t sc3[3] = {hg.y, hg.z, hg.w};
                int sc, mn;
                q4k_scale_min(sc3, jb, sc, mn);
                ag += dg * (float)sc * sx * (float)(128 * cc[0] + cc[1]) - dmg * (float)mn * xm;
            }
            {
                const uint32_t sc3[3] = {hu.y, hu.z, hu.w};
                int sc, mn;
                q4k_scale_min(sc3, jb, sc, mn);
                au += du * (float)sc * sx * (float)(128 * cc[2] + cc[3]) - dmu * (float)mn * xm;
            }
        }
    }
    ag += __shfl_xor_sync(0xffffffffu, ag, 1);
    au += __shfl_xor_sync(0xffffffffu, au, 1);
    ag += __shfl_xor_sync(0xffffffffu, ag, 2);
    au += __shfl_xor_sync(0xffffffffu, au, 2);
    return make_float2(ag, au);
}

// Gate / up rows of a CTA in shared memory, per segment (pairs of one
// expert: top-k slot first, the next slot, the shared expert): its n pairs
// (a multiple of 16) arrive in 8 copies of c = n / 8 consecutive pairs, copy
// m into area m (areas as[s] bytes apart, as[s] % 128 == 32), so pair
// start + m * c + t is row t of area m, and tile t of the segment takes row t
// of every area (8 rows in 8 bank offsets).
struct FdSegs {
    int ns;                                          // segments in use
    int start[3], c[3], off[3], as[3], tile0[3], nt;  // off: byte offset in the gate (and up) region
};
__host__ __device__ __forceinline__ int fd_area_stride(int c, int rb4) {
    const int b = c * rb4;
    return b + ((32 - b % 128) + 128) % 128;
}
__device__ __forceinline__ int fd_seg_of(const FdSegs &S, int i) {
    int s = 0;
    while (s + 1 < S.ns && i >= S.start[s + 1]) s++;
    return s;
}

// Partial dots of the segments' pairs by warps w = 0..NW-1: every tile x
// (NW / tiles) k-parts; part[kp][8 * tile + g] = (gate, up) of row g.
__device__ __noinline__ void pairs_dots(const uint8_t *upg, const uint8_t *upu, const FdSegs *Sp, int rb4,
                                        const unsigned char *xq7, int D, float2 *part, int w, int NW, int lane) {
    const FdSegs &S = *Sp;
    const int nt = S.nt, KP = nt >= NW ? 1 : NW / nt, nb = D / QK;
    for (int it = w; it < nt * KP; it += NW) {
        const int T = it % nt, kp = it / nt;
        int s = 0;
        while (s + 1 < S.ns && T >= S.tile0[s + 1]) s++;
        const size_t o = (size_t)S.off[s] + (size_t)(T - S.tile0[s]) * rb4;
        const float2 r = tile_dots(upg + o, upu + o, S.as[s], kp * nb / KP, (kp + 1) * nb / KP, xq7, D, lane);
        if ((lane & 3) == 0) part[kp * 8 * nt + 8 * T + (lane >> 2)] = r;
    }
}
// h of pair i (index in the segments' numbering) from the k-part partials
// (after a barrier over the NW warps).
__device__ __forceinline__ float pair_h(const float2 *part, const FdSegs &S, int NW, int i) {
    const int nt = S.nt, KP = nt >= NW ? 1 : NW / nt;
    const int s = fd_seg_of(S, i), li = i - S.start[s], g = li / S.c[s], T = S.tile0[s] + li - g * S.c[s];
    float gs = 0.f, us = 0.f;
    for (int kp = 0; kp < KP; kp++) {
        const float2 v = part[kp * 8 * nt + 8 * T + g];
        gs += v.x;
        us += v.y;
    }
    return silu_ref_d(gs) * us;
}

// 32-bit shared-memory loads by shared-window address (ordinary loads, so
// the compiler may schedule them early; barriers and mbarrier waits carry
// memory clobbers).
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    return *reinterpret_cast<const uint32_t *>(__cvta_shared_to_generic(a));
}
// N consecutive 32-bit words starting at a 2-byte aligned shared address.
template <int N>
__device__ __forceinline__ void lds_run2(uint32_t a, uint32_t (&w)[N]) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    uint32_t prev = lds32(b);
#pragma unroll
    for (int i = 0; i < N; i++) {
        const uint32_t nx = lds32(b + 4 * (i + 1));
        w[i] = __funnelshift_r(prev, nx, sh);
        prev = nx;
    }
}

// Quantised h of one expert slot in shared memory: hi / lo byte planes of
// the integer h_int = 256 * hi + lo (h ~= s_g * h_int, per 16-element group
// g), the group scales s_g and the group sums of h_int.
struct HSlot {
    int8_t *hh;
    uint8_t *hl;
    float *hs;
    int *hsum;
};
// Each plane keeps the 128 values of a Q6_K half block in FD_HBS bytes, so
// the half blocks of a plane start in different shared-memory banks.
constexpr int FD_HBS = 144;
__host__ __device__ __forceinline__ int hslot_bytes(int H) { return 2 * (H / 128) * FD_HBS + H / 2; }
__device__ __forceinline__ HSlot hslot(uint8_t *base, int H, int k) {
    uint8_t *p = base + (size_t)k * hslot_bytes(H);
    const int pl = (H / 128) * FD_HBS;
    return HSlot{reinterpret_cast<int8_t *>(p), p + pl, reinterpret_cast<float *>(p + 2 * pl),
                 reinterpret_cast<int *>(p + 2 * pl + H / 4)};
}
// Quantises one 16-row h group (lanes 0..15 hold one value each; lanes
// 16..31 only take part in the shuffles): h_int = rn(h * 32767 / max|h|) =
// 256 * hi + lo (hi int8, lo 0..255), scale max|h| / 32767, and the sum of
// h_int, as HSlot holds them. Stages
// it in shared memory and lets lane 0 store it to group g of the global slot
// image (hslot layout) and count it: its stores, one fence, one add, so the
// count releases exactly the bytes it covers.
__device__ __noinline__ void publish_group(float v, uint8_t *stage, uint8_t *slot, int H, int g, unsigned *count,
                                           int lane) {
    FD_MARK_IF(threadIdx.x == 0, 56)
    if (lane >= 16) v = 0.f;
    float m = fabsf(v);
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = (m > 0.f) ? 32767.0f / m : 0.f;
    const int xi = __float2int_rn(v * inv);
    int sum = xi;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane < 16) {
        stage[lane] = (uint8_t)((xi >> 8) & 0xFF);
        stage[16 + lane] = (uint8_t)(xi & 0xFF);
    }
    __syncwarp();
    if (lane == 0) {
        const uint4 hh = *reinterpret_cast<const uint4 *>(stage), hl = *reinterpret_cast<const uint4 *>(stage + 16);
        const int pl = (H / 128) * FD_HBS, at = (g >> 3) * FD_HBS + (g & 7) * 16;
        *reinterpret_cast<uint4 *>(slot + at) = hh;
        *reinterpret_cast<uint4 *>(slot + pl + at) = hl;
        reinterpret_cast<float *>(slot + 2 * pl)[g] = m / 32767.0f;
        reinterpret_cast<int *>(slot + 2 * pl + H / 4)[g] = sum;
        FD_MARK_IF(threadIdx.x == 0, 54)
        ax::count_add_release(count, 1u);
        FD_MARK_IF(threadIdx.x == 0, 55)
    }
    __syncwarp();
}

// Dot product of one half block (128 weights) of a Q6_K row in shared memory
// (blk = block start, 2-byte aligned shared address) with the quantised h of
// the same 128 positions (hb = half-block index within the row).
__device__ __noinline__ float q6k_half_dot(uint32_t blk, int half, const HSlot &s, int hb) {
    uint32_t ql[16], qh[8], sc[2], dw[1];
    lds_run2<16>(blk + half * 64, ql);
    lds_run2<8>(blk + 128 + half * 32, qh);
    lds_run2<2>(blk + 192 + half * 8, sc);
    lds_run2<1>(blk + 208, dw);
    const int8_t *hh = s.hh + hb * FD_HBS;
    const uint8_t *hl = s.hl + hb * FD_HBS;
    int ahi[8], alo[8];
#pragma unroll
    for (int i = 0; i < 8; i++) ahi[i] = alo[i] = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const uint4 H0 = *reinterpret_cast<const uint4 *>(hh + q * 32);
        const uint4 H1 = *reinterpret_cast<const uint4 *>(hh + q * 32 + 16);
        const uint4 L0 = *reinterpret_cast<const uint4 *>(hl + q * 32);
        const uint4 L1 = *reinterpret_cast<const uint4 *>(hl + q * 32 + 16);
#pragma unroll
        for (int st = 0; st < 8; st++) {
            const uint32_t w = (q & 1) ? ql[8 + st] : ql[st];
            const uint32_t nib = (q & 2) ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu);
            const uint32_t top = ((qh[st] >> (2 * q)) & 0x03030303u) << 4;
            const uint32_t qv = nib | top;
            const int g = q * 2 + (st >> 2);
            const uint32_t hw = comp(st < 4 ? H0 : H1, st & 3), lw = comp(st < 4 ? L0 : L1, st & 3);
            ahi[g] = dp4a_s((int)qv, (int)hw, ahi[g]);
            alo[g] = dp4a_u(qv, lw, alo[g]);
        }
    }
    const float4 s0 = *reinterpret_cast<const float4 *>(s.hs + hb * 8);
    const float4 s1 = *reinterpret_cast<const float4 *>(s.hs + hb * 8 + 4);
    const int4 z0 = *reinterpret_cast<const int4 *>(s.hsum + hb * 8);
    const int4 z1 = *reinterpret_cast<const int4 *>(s.hsum + hb * 8 + 4);
    const float hsv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const int hzv[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
    float y = 0.f;
#pragma unroll
    for (int g = 0; g < 8; g++) {
        const int scale = (int)(int8_t)((g < 4 ? sc[0] : sc[1]) >> (8 * (g & 3)));
        const int S = ahi[g] * 256 + alo[g] - 32 * hzv[g];
        y += (float)scale * hsv[g] * (float)S;
    }
    return half_bits_ref(dw[0] & 0xFFFFu) * y;
}

__global__ void __launch_bounds__(FD_THREADS, 1) decode_fused_kernel(FusedDecodeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const FusedPlan &P = a.p;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int D = a.D, H = a.H, E = a.E, K = a.K;
    const int rb4 = (D / QK) * Q4K_BYTES, rb6 = (H / QK) * Q6K_BYTES;
    const size_t exp4 = (size_t)rb4 * H, exp6 = (size_t)rb6 * D;

    float *xs = reinterpret_cast<float *>(sm + P.o_x);
    unsigned char *xq = sm + P.o_xq;
    float *rrow = reinterpret_cast<float *>(sm + P.o_rr);
    float *hbuf = reinterpret_cast<float *>(sm + P.o_hb);  // h of my row slots (routed, then shared)
    float2 *part = reinterpret_cast<float2 *>(sm + P.o_part);  // k-part partial dots (pairs_dots)
    uint8_t *hst = sm + P.o_hst;                            // [FD_WARPS][FD_GROUP_BYTES] staging
    uint8_t *hqg = reinterpret_cast<uint8_t *>(a.hll);      // global image of the quantised h slots
    const int SLOT = hslot_bytes(H);                         // bytes per slot (hslot layout)
    uint8_t *dn = sm + P.o_dn;  // slot K (shared) first, then routed slots 0..K-1
    uint8_t *upg = sm + P.o_up;
    uint8_t *upu = upg + P.upb;  // up rows: the same layout as the gate rows
    uint8_t *hqb = sm + P.o_hq;
    float *Lf = reinterpret_cast<float *>(sm + P.o_sel);
    float *Bf = Lf + E;
    float *ysp = reinterpret_cast<float *>(sm + P.o_ys);  // [K+1][rows_cap][NHB] partial dots
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.o_bar);
    uint64_t *mb_pre = bars, *mb_x = bars + 1, *mb_up = bars + 2, *mb_dn = bars + 4;  // mb_dn[K]
    uint64_t *mb_h = bars + 4 + K;  // the copy of every routed h (step 4)
    const int nbars = 5 + K;
    const size_t sdn = P.sdn;      // shared bytes per slot of down rows
    const int rows_cap = P.ngc;    // output rows per CTA at most
    const int NHB = H / 128;       // half blocks per Q6_K row
    auto dnp = [&](int k) { return dn + (size_t)(k == K ? 0 : k + 1) * sdn; };

    __shared__ int s_top[16];
    __shared__ float s_w[16];
    __shared__ uint32_t s_tag, s_par;
    __shared__ int s_mode, s_nc, s_full, s_wcnt[FD_WARPS];
    __shared__ float s_max, s_sum, s_gsc;
    __shared__ double s_lo;
    __shared__ uint32_t s_err;

    // ---- work shares of this CTA ----
    const int nrows = E + a.use_gate;
    const int nr_mine = c < nrows ? (nrows - 1 - c) / G + 1 : 0;  // rows c, c+G, ...
    const int NRG = K * H / 16, NSG = a.has_shared ? H / 16 : 0;  // routed / shared h groups
    const FdShare share = fd_share(c, G, NRG, NSG);
    const int u0 = 16 * share.rg0, u1 = 16 * share.rg1;  // routed pairs, top-k slot order
    const int s0 = 16 * share.sg0, s1 = 16 * share.sg1;  // shared-expert rows
    const int nrp = u1 - u0;                              // row slots [0, nrp) routed, then shared
    // output rows [n0, n1), as even as rows go; the down slabs are copied
    // from a0 = n0 rounded down to dg rows (16-byte aligned), their size
    // rounded up to 16 bytes (the rows past n1 are never read)
    const int n0 = (int)((long long)c * D / G), n1 = (int)((long long)(c + 1) * D / G);
    const int nrow_out = n1 - n0, a0 = n0 - n0 % P.dg;
    const uint32_t slab = (uint32_t)(((n1 - a0) * rb6 + 15) & ~15);
    const int slot_first = u0 / H;  // the CTA's pairs span slots slot_first and (maybe) slot_first + 1
    // row segments: routed pairs of slot_first, of slot_first + 1, then the
    // shared-expert rows (s_seg[0] routed, s_seg[1] shared)
    __shared__ FdSegs s_seg[2];
    if (tid == 0) {
        const int n0s = min(u1, (slot_first + 1) * H) - u0, ns = s1 - s0;
        const int n[3] = {n0s, nrp - n0s, ns};
        int off = 0;
        for (int q = 0; q < 3; q++) {
            FdSegs &S = s_seg[q < 2 ? 0 : 1];
            const int j = q < 2 ? q : 0;
            if (j == 0) { S.ns = 0; S.nt = 0; }
            if (n[q] == 0) continue;
            const int cq = n[q] / 8, asq = fd_area_stride(cq, rb4);
            S.start[S.ns] = q == 2 ? 0 : (q == 0 ? 0 : n0s);
            S.c[S.ns] = cq;
            S.off[S.ns] = off;
            S.as[S.ns] = asq;
            S.tile0[S.ns] = S.nt;
            S.nt += cq;
            S.ns++;
            off += 8 * asq;
        }
    }
    // (s_seg is published by the __syncthreads after the mbarrier set-up)

    // Copies of top-k slot q (expert e): my gate/up rows inside slot q and my
    // output rows' down slab. One arrival on each mbarrier per issue round.
    // Routed copies: per segment 8 copies per matrix (FdSegs); expect_up
    // announces each segment's bytes once (slot_first, slot_first + 1).
    auto expect_up = [&]() {
        const int sb = min(u1, (slot_first + 1) * H);
        ax::mbar_arrive_expect(mb_up, 2u * (uint32_t)(sb - u0) * rb4);
        ax::mbar_arrive_expect(mb_up + 1, 2u * (uint32_t)(u1 - sb) * rb4);
    };
    // copy v (0..31) of the routed rows: segment v / 16, matrix (v / 8) & 1, area v & 7
    auto issue_rows = [&](int v0, int step) {
        const FdSegs &S = s_seg[0];
        for (int v = v0; v < 16 * S.ns; v += step) {
            const int sg = v >> 4, mat = (v >> 3) & 1, m = v & 7;
            const int p = u0 + S.start[sg] + m * S.c[sg], q = p / H;
            uint64_t *b = mb_up + (q == slot_first ? 0 : 1);
            const size_t src = (size_t)s_top[q] * exp4 + (size_t)(p - q * H) * rb4;
            ax::bulk_g2s_hint((mat ? upu : upg) + S.off[sg] + (size_t)m * S.as[sg], (mat ? a.up : a.gate) + src,
                              (uint32_t)S.c[sg] * rb4, b, ax::l2_evict_first());
        }
    };
    auto issue_dn = [&](int q, int e) {
        ax::mbar_arrive_expect(mb_dn + q, nrow_out ? slab : 0u);
        if (nrow_out)
            ax::bulk_g2s_hint(dnp(q), a.down + (size_t)e * exp6 + (size_t)a0 * rb6, slab, mb_dn + q, ax::l2_evict_first());
    };

    // ---- step 0: static bytes, before waiting for the producer of x ----
    FD_MARK(0)
    if (tid == 0) {
        s_err = 0;
        s_par = 0;
        for (int i = 0; i < nbars; i++) ax::mbar_init(bars + i, 1);
        ax::mbar_init_fence();
    }
    __syncthreads();
    pdl_trigger();
    if (tid == 0) {
        uint32_t bytes = (uint32_t)nr_mine * D * 4;
        if (a.has_shared) bytes += 2u * (s1 - s0) * rb4 + (nrow_out ? slab : 0u);
        ax::mbar_arrive_expect(mb_pre, bytes);
        for (int i = 0; i < nr_mine; i++) {
            const int r = c + i * G;
            const float *src = r < E ? a.W + (size_t)r * D : a.gate_v;
            ax::bulk_g2s(rrow + (size_t)i * D, src, D * 4, mb_pre);
        }
        if (a.has_shared) {
            if (s1 > s0) {
                const FdSegs &S = s_seg[1];
                for (int m = 0; m < 8; m++) {
                    const size_t src = (size_t)(s0 + m * S.c[0]) * rb4, dst = S.off[0] + (size_t)m * S.as[0];
                    ax::bulk_g2s(upg + dst, a.gate_sh + src, (uint32_t)S.c[0] * rb4, mb_pre);
                    ax::bulk_g2s(upu + dst, a.up_sh + src, (uint32_t)S.c[0] * rb4, mb_pre);
                }
            }
            if (nrow_out) ax::bulk_g2s(dnp(K), a.down_sh + (size_t)a0 * rb6, slab, mb_pre);
        }
    }
    pdl_wait();
    FD_MARK(1)
    // the residual of my output rows, read now (used by the combine)
    float *res_s = reinterpret_cast<float *>(sm + P.o_res);
    if (tid < nrow_out) res_s[tid] = a.resid ? a.resid[n0 + tid] : 0.f;
    if (tid == 0) {
        s_tag = *reinterpret_cast<volatile unsigned int *>(a.sync) + 1u;
        ax::mbar_arrive_expect(mb_x, D * 4);
        ax::bulk_g2s(xs, a.x, D * 4, mb_x);
    }
    bool tag_fail = false, copy_fail = false;
    if (!ax::mbar_wait(mb_x, 0, FD_WAIT_NS)) copy_fail = true;
    if (!ax::mbar_wait(mb_pre, 0, FD_WAIT_NS)) copy_fail = true;
    __syncthreads();
    const uint32_t tag = s_tag;
    FD_MARK(2)

    // ---- step 1: router rows (published first) ----
    {
        // tpr threads per router row (wpr warps): thread lt owns elements
        // [lt*seg, lt*seg+seg), seg >= 4, and forms (P = its sum, SP = sum of
        // |prefix| inside the segment, A = sum of |product|). The row's
        // prefix before each segment comes from a warp scan plus the totals
        // of the row's earlier warps; S_P <= sum over segments of
        // seg*|prefix before| + SP.
        const int tpr = D % 1024 == 0 ? 256 : D / 4, seg = D / tpr, wpr = tpr / 32;
        const int ri = tid / tpr, lt = tid - ri * tpr, wr = lt >> 5;
        const bool mine = ri < nr_mine;
        // scratch: the routed down slabs, filled only after the selection
        double *wtot = reinterpret_cast<double *>(dn + sdn);  // [rmax][wpr] warp sums of P
        double *wsa = wtot + P.rmax * wpr;                    // [rmax][wpr][2] warp sums of (S_P bound, A)
        double Pd = 0.0, SPd = 0.0, Ad = 0.0;
        if (mine) {
            const float *w = rrow + (size_t)ri * D + lt * seg;
            const float *xv = xs + lt * seg;
            // products exact as (p, e) pairs (fma), summed as a float pair
            // (two-sum): the running sum is exact to ~2^-44 of sum|p|, far
            // inside the bound's 2^-9 slack; |prefix| and |p| sums in fp32
            // are upper bounds within a few ulps (same slack)
            float hi = 0.f, lo = 0.f, SPf = 0.f, Af = 0.f;
            for (int i = 0; i < seg; i += 4) {
                const float4 w4 = *reinterpret_cast<const float4 *>(w + i);
                const float4 x4 = *reinterpret_cast<const float4 *>(xv + i);
                const float xx[4] = {x4.x, x4.y, x4.z, x4.w}, ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float p = __fmul_rn(xx[k], ww[k]), e = __fmaf_rn(xx[k], ww[k], -p);
                    const float sm = __fadd_rn(hi, p), bb = __fsub_rn(sm, hi);
                    const float er = __fadd_rn(__fsub_rn(hi, __fsub_rn(sm, bb)), __fsub_rn(p, bb));
                    hi = sm;
                    lo = __fadd_rn(lo, __fadd_rn(er, e));
                    SPf = __fadd_ru(SPf, fabsf(__fadd_rn(hi, lo)));
                    Af = __fadd_ru(Af, fabsf(p));
                }
            }
            Pd = (double)hi + (double)lo;
            SPd = (double)SPf * (1.0 + 0x1.0p-20);
            Ad = (double)Af * (1.0 + 0x1.0p-20);
        }
        FD_MARK(20)
        double inc = Pd;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double up = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += up;
        }
        if (mine && lane == 31) wtot[ri * wpr + wr] = inc;
        __syncthreads();
        FD_MARK(21)
        double base = 0.0, L = 0.0;
        if (mine)
            for (int q = 0; q < wpr; q++) {
                const double v = wtot[ri * wpr + q];
                if (q < wr) base += v;
                L += v;
            }
        double spb = (double)seg * fabs(base + inc - Pd) + SPd, At = Ad;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            spb += __shfl_xor_sync(0xffffffffu, spb, o);
            At += __shfl_xor_sync(0xffffffffu, At, o);
        }
        if (mine && lane == 0) {
            wsa[2 * (ri * wpr + wr)] = spb;
            wsa[2 * (ri * wpr + wr) + 1] = At;
        }
        ax::fence_proxy_async_smem();  // this area is refilled by bulk copies after the selection
        __syncthreads();
        FD_MARK(22)
        if (mine && lt == 0) {
            spb = 0.0;
            At = 0.0;
            for (int q = 0; q < wpr; q++) {
                spb += wsa[2 * (ri * wpr + q)];
                At += wsa[2 * (ri * wpr + q) + 1];
            }
            ax::fence_proxy_async_smem();  // (those reads) before the bulk copies that refill it
            const int r = c + ri * G;
            FD_MARK(23)
            if (r < E) {
                const double Bd = a.bound_scale * (At + spb + a.ngam * At) + 0x1.0p-60;
                const float lf = __double2float_rn(L);
                const float bf = __double2float_ru(Bd + fabs(L - (double)lf));
                ax::put_tagged(a.cand + 2 * r, u_of(lf), tag);
                ax::put_tagged(a.cand + 2 * r + 1, u_of(bf), tag);
            } else {
                ax::put_tagged(a.cand + 2 * E, u_of(1.0f / (1.0f + expf(-(float)L))), tag);
            }
            // relaxed: the count only says when to read; a reader that sees
            // it before a word's store polls that word until its tag matches
            ax::count_add_relaxed(a.sync + 3, 1u);
        }
    }
    FD_MARK(3)

    // ---- step 2: two warp groups until the selection is known ----
    // group A (warps 0-7): all (L~, B) -> warp 0 selects the top-k, issues the
    //   routed copies and certifies; group B (warps 8-15): quantised x, the
    //   shared expert's h rows, then its down rows.
    constexpr int GRP = FD_THREADS / 2;
    if (tid < GRP) {
        // one thread waits for the count of published rows, then every
        // thread reads its entries once (no polling storm on these lines)
        // (the shared gate's logit is counted with the router rows)
        if (tid == 0 && !ax::wait_count(a.sync + 3, tag * (unsigned)nrows, FD_WAIT_NS)) tag_fail = true;
        asm volatile("bar.sync 1, %0;" ::"r"(GRP) : "memory");
        for (int e = tid; e < E; e += GRP) {
            uint32_t v0, v1;
            if (!ax::get_tagged2(a.cand + 2 * e, tag, v0, v1, FD_WAIT_NS)) tag_fail = true;
            Lf[e] = f_of(v0);
            Bf[e] = f_of(v1);
        }
        if (tid == GRP - 1)
            s_gsc = a.use_gate ? f_of(ax::get_tagged(a.cand + 2 * E, tag, FD_WAIT_NS, tag_fail)) : 1.0f;
        asm volatile("bar.sync 1, %0;" ::"r"(GRP) : "memory");
        FD_MARK(6)
        if (wid != 0) {
            // copy v: routed gate/up row copies [0, 16 * ns), then the down
            // slab of slot v - 16 * ns; warp w (1..7), lane l takes v = 7 l + w - 1
            asm volatile("bar.sync 3, %0;" ::"r"(GRP) : "memory");
            const int nv = 16 * s_seg[0].ns, v = 7 * lane + wid - 1;
            if (v < nv) issue_rows(v, nv);
            else if (v < nv + K) issue_dn(v - nv, s_top[v - nv]);
        }
        if (wid == 0) {
            // keys: the order-preserving bits of L~ truncated to 24 bits, then
            // 255 - e (a larger key wins; equal values go to the smaller
            // index). The truncation can only mis-order logits closer than
            // 2^-15 relative; the certificate below checks the chosen order
            // on the full values, so such a choice is never certified.
            uint32_t k8[FD_PER_LANE];
#pragma unroll
            for (int j = 0; j < FD_PER_LANE; j++) {
                const int e = lane + 32 * j;
                const uint32_t u = e < E ? __float_as_uint(Lf[e]) : 0u;
                const uint32_t ok = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
                k8[j] = e < E ? ((ok & 0xFFFFFF00u) | (uint32_t)(255 - e)) : 0u;
            }
            // sort each lane's 8 keys descending (19-comparator network)
            auto cx = [&](int p, int q) { const uint32_t hi = max(k8[p], k8[q]), lo = min(k8[p], k8[q]); k8[p] = hi; k8[q] = lo; };
            cx(0, 2); cx(1, 3); cx(4, 6); cx(5, 7);
            cx(0, 4); cx(1, 5); cx(2, 6); cx(3, 7);
            cx(0, 1); cx(2, 3); cx(4, 5); cx(6, 7);
            cx(2, 4); cx(3, 5);
            cx(1, 4); cx(3, 6);
            cx(1, 2); cx(3, 4); cx(5, 6);
            FD_MARK(30)
            int my_e = 0;
            for (int q = 0; q < K; q++) {
                const uint32_t wk = __reduce_max_sync(0xffffffffu, k8[0]);
                if (k8[0] == wk) {
#pragma unroll
                    for (int j = 0; j < FD_PER_LANE - 1; j++) k8[j] = k8[j + 1];
                    k8[FD_PER_LANE - 1] = 0u;
                }
                if (lane == q) my_e = 255 - (int)(wk & 0xFFu);
            }
            // every lane issues gate / up rows, lane q < K slot q's down slab
            FD_MARK(31)
            if (lane < K) s_top[lane] = my_e;
            __syncwarp();
            if (lane == 0) expect_up();
            // warps 1-7 issue the copies (a warp issues its lanes' bulk
            // copies one after another, so spreading them shortens the issue)
            asm volatile("bar.arrive 3, %0;" ::"r"(GRP) : "memory");
            FD_MARK(16)
            // certificate: every adjacent gap inside the top-k and the gap to
            // the rest exceed both bounds plus the margin (rounded against success)
            float hi_rest = -INFINITY;
#pragma unroll
            for (int j = 0; j < FD_PER_LANE; j++)
                if (k8[j]) {
                    const int e = 255 - (int)(k8[j] & 0xFFu);
                    hi_rest = fmaxf(hi_rest, __fadd_ru(Lf[e], Bf[e]));
                }
            hi_rest = fmaxf(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, 16));
            hi_rest = fmaxf(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, 8));
            hi_rest = fmaxf(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, 4));
            hi_rest = fmaxf(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, 2));
            hi_rest = fmaxf(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, 1));
            const float myL = lane < K ? Lf[my_e] : 0.f, myB = lane < K ? Bf[my_e] : 0.f;
            const float nL = __shfl_down_sync(0xffffffffu, myL, 1), nB = __shfl_down_sync(0xffffffffu, myB, 1);
            const float L0 = __shfl_sync(0xffffffffu, myL, 0);
            bool ok = true;
            if (lane < K) {
                const float nxt = lane + 1 < K ? __fadd_ru(nL, nB) : hi_rest;
                ok = __fsub_rd(myL, myB) > __fadd_ru(nxt, (float)FD_MARGIN);
                if (lane == K - 1) ok = ok && (myL - L0 > -80.0f);
            }
            ok = __all_sync(0xffffffffu, ok);
            if (lane == 0) s_mode = ok ? 0 : 1;
            FD_MARK(17)
            if (ok) {
                // weights: fp32 softmax of L~ (model.c:1027-1049 / :300-316 forms)
                float sum = 0.f;
                if (a.routing == OFB_ROUTE_FORWARD) {
#pragma unroll
                    for (int j = 0; j < FD_PER_LANE; j++)
                        if (lane + 32 * j < E) sum += expf(Lf[lane + 32 * j] - L0);
                } else if (lane < K) {
                    sum = expf(myL - L0);
                }
                sum = warp_sum(sum);
                const float wq = lane < K ? expf(myL - L0) / sum : 0.f;
                const float ss = warp_sum(wq);
                if (lane < K) s_w[lane] = (a.routing == OFB_ROUTE_FORWARD && a.renorm) ? wq / ss : wq;
                FD_MARK(18)
            } else {
                float lo = lane < K ? __fsub_rd(myL, myB) : INFINITY;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                if (lane == 0) s_lo = lo;
            }
        }
    } else {
        const int gt = tid - GRP;  // thread index inside group B
        // quantised x for the tensor-core dots: one lane per 32-element
        // sub-block, no shuffles
        for (int sb = gt; sb < D / 32; sb += GRP) {
            const float4 *v4 = reinterpret_cast<const float4 *>(xs + sb * 32);
            float v[32];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 t = v4[i];
                v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
            }
            float m = 0.f, xsum = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i++) { m = fmaxf(m, fabsf(v[i])); xsum += v[i]; }
            // x_int = rn(x * 16383 / max|x|) = 128 * hi + lo, hi int8, lo 0..127
            const float s = m / 16383.0f, inv = (m > 0.0f) ? 16383.0f / m : 0.0f;
            uint32_t hw[8], lw[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                uint32_t h4 = 0, l4 = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int xi = __float2int_rn(v[4 * q + i] * inv);
                    h4 |= ((uint32_t)(xi >> 7) & 0xFFu) << (8 * i);
                    l4 |= ((uint32_t)xi & 0x7Fu) << (8 * i);
                }
                hw[q] = h4;
                lw[q] = l4;
            }
            uint4 *qh4 = reinterpret_cast<uint4 *>(xq + sb * 32), *ql4 = reinterpret_cast<uint4 *>(xq + D + sb * 32);
            qh4[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            qh4[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            ql4[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            ql4[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
            reinterpret_cast<float *>(xq + 2 * D)[sb] = s;
            reinterpret_cast<float *>(xq + 2 * D)[D / 32 + sb] = xsum;
        }
        asm volatile("bar.sync 2, %0;" ::"r"(GRP) : "memory");
        FD_MARK_IF(gt == 0, 4)
        if (a.has_shared && s1 > s0) {
            // my shared-expert rows (row slots nrp..) on the tensor cores,
            // then each 16-row group quantised and published to slot K
            const int gw = wid - GRP / 32, NW = GRP / 32, ns = s1 - s0;
            pairs_dots(upg, upu, &s_seg[1], rb4, xq, D, part, gw, NW, lane);
            asm volatile("bar.sync 2, %0;" ::"r"(GRP) : "memory");
            for (int i = gt; i < ns; i += GRP) hbuf[nrp + i] = pair_h(part, s_seg[1], NW, i);
            asm volatile("bar.sync 2, %0;" ::"r"(GRP) : "memory");
            FD_MARK_IF(gt == 0, 5)
            for (int g = gw; g < ns / 16; g += NW)
                publish_group(hbuf[nrp + 16 * g + (lane & 15)], hst + wid * FD_GROUP_BYTES, hqg + (size_t)K * SLOT, H,
                              share.sg0 + g, a.sync + 4, lane);
            FD_MARK_IF(gt == 0, 29)
        }
    }
    __syncthreads();
    FD_MARK(7)
    if (s_mode != 0) {
        // ---- uncertain: the reference's exact chain for the candidates ----
        // The scratch overlays the routed down slabs and gate/up rows: let the
        // copies already issued land, and issue the final ones afterwards.
        if (tid == 0)
            for (int i = 2; i < 4 + K; i++)  // mb_up, mb_dn (not mb_h: step 4)
                if (!ax::mbar_wait(bars + i, 0, FD_WAIT_NS)) copy_fail = true;
        __syncthreads();
        float *wbuf = reinterpret_cast<float *>(dn + sdn);
        float *val = reinterpret_cast<float *>(dn + sdn + XL_SMEM);
        int *id = reinterpret_cast<int *>(val + E);
        float *oval = reinterpret_cast<float *>(id + E);
        int *oid = reinterpret_cast<int *>(oval + E);
        int *clist = oid + E;
        float *cv = reinterpret_cast<float *>(clist + E);
        int *cid = reinterpret_cast<int *>(cv + E);
        float *cov = reinterpret_cast<float *>(cid + E);
        int *coid = reinterpret_cast<int *>(cov + E);
        int *taken = coid + E;
        const double lo_min = s_lo;
        if (tid == 0) { s_nc = 0; s_full = 0; }
        __syncthreads();
        // candidates in ascending expert order: experts outside the list
        // never win a strict comparison of the exchange sort, so sorting the
        // candidates alone gives the full sort's order
        for (int e0 = 0; e0 < E; e0 += FD_THREADS) {
            const int e = e0 + tid;
            const bool cand = e < E && ((double)Lf[e] + (double)Bf[e] >= lo_min - FD_MARGIN);
            if (e < E) { val[e] = -INFINITY; id[e] = e; taken[e] = cand; }
            const unsigned bal = __ballot_sync(0xffffffffu, cand);
            if (lane == 0) s_wcnt[wid] = __popc(bal);
            __syncthreads();
            int off = s_nc;
            for (int q = 0; q < wid; q++) off += s_wcnt[q];
            if (cand) clist[off + __popc(bal & ((1u << lane) - 1u))] = e;
            __syncthreads();
            if (tid == 0)
                for (int q = 0; q < FD_WARPS; q++) s_nc += s_wcnt[q];
            __syncthreads();
        }
        const int nc = s_nc;
        exact_logits_block(a.W, D, xs, clist, nc, cv, wbuf, tid, FD_THREADS);
        __syncthreads();
        for (int q = tid; q < nc; q += FD_THREADS) {
            val[clist[q]] = cv[q];
            cid[q] = clist[q];
        }
        __syncthreads();
        if (a.routing == OFB_ROUTE_FORWARD) {
            // probabilities order like expf(l - max) unless two of them are
            // within a few ulps (then the division could tie them)
            if (wid == 0) {
                float m = -INFINITY;
                for (int q = lane; q < nc; q += 32) m = fmaxf(m, cv[q]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (lane == 0) s_max = m;
            }
            __syncthreads();
            for (int q = tid; q < nc; q += FD_THREADS) cv[q] = ofb_exact_expf(__fsub_rn(cv[q], s_max));
            __syncthreads();
            for (int q = tid; q < nc; q += FD_THREADS)
                for (int q2 = 0; q2 < nc; q2++)
                    if (q2 != q && close_ulps(cv[q], cv[q2], 4)) s_full = 1;
            __syncthreads();
            if (s_full) {
                // every logit exact, softmax as the reference computes it
                for (int e = tid; e < E; e += FD_THREADS)
                    val[e] = taken[e] ? val[e] : exact_logit(a.W + (size_t)e * D, xs, D);
                __syncthreads();
                if (tid == 0) {
                    float m = val[0];
                    for (int e = 1; e < E; e++) if (val[e] > m) m = val[e];
                    s_max = m;
                }
                __syncthreads();
                for (int e = tid; e < E; e += FD_THREADS) val[e] = ofb_exact_expf(__fsub_rn(val[e], s_max));
                __syncthreads();
                if (tid == 0) {
                    float s = 0.0f;
                    for (int e = 0; e < E; e++) s = __fadd_rn(s, val[e]);
                    s_sum = s;
                }
                __syncthreads();
                for (int e = tid; e < E; e += FD_THREADS) val[e] = __fdiv_rn(val[e], s_sum);
                __syncthreads();
            }
        }
        if (wid == 0) {
            if (s_full) {
                exchange_topk(val, id, oval, oid, E, K, lane);
                if (lane == 0) {
                    float ssum = 0.0f;
                    for (int q = 0; q < K; q++) ssum = __fadd_rn(ssum, val[q]);
                    for (int q = 0; q < K; q++) {
                        s_top[q] = id[q];
                        s_w[q] = a.renorm ? __fdiv_rn(val[q], ssum) : val[q];
                    }
                    s_mode = 2;
                }
            } else {
                exchange_topk(cv, cid, cov, coid, nc, K, lane);
                __syncwarp();
                const int tk = lane < K ? cid[lane] : 0;
                const float m = Lf[cid[0]];
                float sum = 0.f;
                if (a.routing == OFB_ROUTE_FORWARD) {
                    for (int e = lane; e < E; e += 32) sum += expf(Lf[e] - m);
                } else if (lane < K) {
                    sum = expf(Lf[tk] - m);
                }
                sum = warp_sum(sum);
                const float wq = lane < K ? expf(Lf[tk] - m) / sum : 0.f;
                const float ss = warp_sum(wq);
                if (lane < K) {
                    s_top[lane] = tk;
                    s_w[lane] = (a.routing == OFB_ROUTE_FORWARD && a.renorm) ? wq / ss : wq;
                }
            }
        }
        // this memory is refilled by bulk copies next
        ax::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            s_par = 1;
            expect_up();
            issue_rows(0, 1);
            for (int q = 0; q < K; q++) issue_dn(q, s_top[q]);
        }
        __syncthreads();
    }
    if (c == 0 && tid < K) {
        if (a.idx_out) a.idx_out[tid] = (uint32_t)s_top[tid];
        if (a.w_out) a.w_out[tid] = s_w[tid];
        if (tid == 0 && a.stats) atomicAdd(&a.stats[s_mode], 1);
    }
    const uint32_t par = s_par;
    FD_MARK(19)

    // ---- step 3: routed h rows on the tensor cores, every warp (tiles of 8
    // pairs x k-parts), once both segments' rows have landed ----
    {
        const int np = nrp;
        if (!ax::mbar_wait(mb_up, par, FD_WAIT_NS)) copy_fail = true;
        if (!ax::mbar_wait(mb_up + 1, par, FD_WAIT_NS)) copy_fail = true;
        FD_MARK(28)
        pairs_dots(upg, upu, &s_seg[0], rb4, xq, D, part, wid, FD_WARPS, lane);
        FD_MARK(51)
        __syncthreads();
        FD_MARK(8)
        for (int i = tid; i < np; i += FD_THREADS) hbuf[i] = pair_h(part, s_seg[0], FD_WARPS, i);
        __syncthreads();
        FD_MARK(10)
        // each 16-row group quantised once, here, and published to its slot
        for (int g = wid; g < np / 16; g += FD_WARPS) {
            const int rg = u0 / 16 + g, k = rg / (H / 16), gs = rg - k * (H / 16);
            publish_group(hbuf[16 * g + (lane & 15)], hst + wid * FD_GROUP_BYTES, hqg + (size_t)k * SLOT, H, gs,
                          a.sync + 4, lane);
        }
    }
    // every CTA has published everything it publishes in this launch: count
    // it finished (off the critical path: the h groups of the other CTAs are
    // still arriving). The last one sets the exchange counters to their exact
    // values for this epoch (repairing them after an expired wait) and
    // advances the epoch; every CTA read the epoch before publishing its
    // router rows, and nothing reads it again in this launch.
    __syncthreads();
    if (tid == 32) {
        if (ax::count_add_acq_rel(&a.sync[1], 1u) == (unsigned)G - 1) {
            a.sync[1] = 0;
            a.sync[3] = tag * (unsigned)nrows;
            a.sync[4] = tag * (unsigned)(NRG + NSG);
            __threadfence();
            atomicAdd(&a.sync[0], 1u);
        }
    }
    FD_MARK(9)
    // ---- step 4: the quantised h of every slot (one bulk copy of the
    // global slot image once every group is counted); y of my rows ----
    const int nslot = K + (a.has_shared ? 1 : 0);
    if (tid == 0) {
        if (!ax::wait_count(a.sync + 4, tag * (unsigned)(NRG + NSG), FD_WAIT_NS)) tag_fail = true;
        FD_MARK(26)
        ax::fence_proxy_async_global();  // the acquired groups, seen by the copy
        ax::mbar_arrive_expect(mb_h, (uint32_t)nslot * SLOT);
        ax::bulk_g2s(hqb, hqg, (uint32_t)nslot * SLOT, mb_h);
    }
    if (!ax::mbar_wait(mb_h, 0, FD_WAIT_NS)) copy_fail = true;
    FD_MARK(11)
    // the routed slots and (slot K) the shared expert: one task per thread at
    // the BASELINE shape
    for (int t = tid; t < nslot * nrow_out * NHB; t += FD_THREADS) {
        const int kh = t / nrow_out, r = t - kh * nrow_out, k = kh / NHB, hb = kh - k * NHB;
        if (k < K && !ax::mbar_wait(mb_dn + k, par, FD_WAIT_NS)) copy_fail = true;
        const uint32_t base = ax::smem_u32(dnp(k)) + (n0 - a0) * rb6;
        ysp[((size_t)k * rows_cap + r) * NHB + hb] =
            q6k_half_dot(base + r * rb6 + (hb >> 1) * Q6K_BYTES, hb & 1, hslot(hqb, H, k), hb);
    }
    FD_MARK(12)
    __syncthreads();
    FD_MARK(13)
    // y per (slot, row): the half-block partials summed in a fixed order,
    // into the first partial's place
    for (int t = tid; t < (K + 1) * nrow_out; t += FD_THREADS) {
        const int k = t / nrow_out, r = t - k * nrow_out;
        float *pp = ysp + ((size_t)k * rows_cap + r) * NHB;
        float v = 0.f;
        for (int hb = 0; hb < NHB; hb++) v += pp[hb];
        pp[0] = v;
    }
    __syncthreads();
    for (int r = tid; r < nrow_out; r += FD_THREADS) {
        const int n = n0 + r;
        float acc = res_s[r];  // thread r wrote it after the dependent-launch wait
        float yv[16], wv[16];
#pragma unroll
        for (int k = 0; k < 16; k++) {
            yv[k] = k < K ? ysp[((size_t)k * rows_cap + r) * NHB] : 0.f;
            wv[k] = k < K ? s_w[k] : 0.f;
        }
        if (a.has_shared) {
            const float y = ysp[((size_t)K * rows_cap + r) * NHB];
            acc += a.use_gate ? s_gsc * y : y;
        }
        float rr = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++)
            if (k < K && !(wv[k] < 1e-6f)) rr += wv[k] * yv[k];  // model.c:1066 skip rule
        a.out[n] = acc + rr;
    }
    FD_MARK(14)

    // ---- exit: errors, copies in flight, epoch ----
    if (copy_fail || tag_fail) atomicOr(&s_err, (copy_fail ? FD_ERR_COPY : 0u) | (tag_fail ? FD_ERR_TAG : 0u));
    __syncthreads();
    if (tid == 0) {
        if (s_err) {
            atomicOr(&a.sync[2], s_err);
            // let every copy this CTA issued land before its shared memory goes
            for (int i = 0; i < nbars; i++) ax::mbar_wait(bars + i, (i < 2 || i == nbars - 1) ? 0 : par, FD_WAIT_NS);
        }
    }
    FD_MARK(15)
}

// ---- host ----------------------------------------------------------------------
#ifdef OFB_FD_TRACE
extern "C" int ofb_debug_fd_trace(unsigned long long *host) {
    return cudaMemcpyFromSymbol(host, g_fd_tr, sizeof(g_fd_tr)) == cudaSuccess ? 0 : 1;
}
#endif

static int gcd_i(int a, int b) { return b ? gcd_i(b, a % b) : a; }

bool fused_plan(const ofb_moe_config *cfg, bool use_gate, bool has_shared, int G, FusedPlan &p) {
    const int D = cfg->d_model, H = cfg->hidden, E = cfg->n_experts, K = cfg->top_k;
    if (E > 32 * FD_PER_LANE || K > 16 || K > E || G < 1 || H % 16) return false;
    const int nrows = E + (use_gate ? 1 : 0);
    p.G = G;
    p.rmax = (nrows + G - 1) / G;
    const int tpr = D % 1024 == 0 ? 256 : D / 4;
    if (tpr > FD_THREADS || p.rmax > FD_THREADS / tpr) return false;
    const int nbk = H / QK, rb4 = (D / QK) * Q4K_BYTES, rb6 = nbk * Q6K_BYTES;
    // output rows per group: 16-byte aligned Q6_K slabs (dg * rb6 % 16 == 0)
    int dg = 8 / gcd_i(nbk, 8);
    if (dg < 4) dg = 4;
    if (D % dg) return false;
    p.dg = dg;
    // gate/up row slots: the CTA's routed pairs, then its shared-expert rows
    const int NR = K * H / 16, NS = has_shared ? H / 16 : 0;
    int most = 0, most_r = 0;
    for (int c = 0; c < G; c++) {
        const FdShare sh = fd_share(c, G, NR, NS);
        most = std::max(most, sh.rg1 - sh.rg0 + sh.sg1 - sh.sg0);
        most_r = std::max(most_r, sh.rg1 - sh.rg0);
    }
    p.upc = 16 * most;
    // gate (and up) region: up to three segments of 8 areas, each padded to
    // a bank offset of 32 bytes
    p.upb = (uint32_t)(((size_t)p.upc * rb4 + 24 * 128 + 127) & ~(size_t)127);
    if (16 * most_r > H) return false;  // a CTA's routed pairs span at most two slots
    p.ngc = (D + G - 1) / G;  // output rows per CTA at most
    const int rows_cap = p.ngc;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = (off + bytes + 127) & ~(size_t)127; return (uint32_t)o; };
    p.o_x = take((size_t)D * 4);
    p.o_xq = take(xq_stride(D));
    p.o_rr = take((size_t)p.rmax * D * 4);
    // down slabs (shared expert first, then the routed slots) directly
    // followed by the gate/up rows: the router rows' partial sums use the
    // routed down slabs before they are filled, and the selection's
    // exact-recompute scratch overlays the routed part of both
    const size_t sdn = ((size_t)(rows_cap + dg - 1) * rb6 + 15) & ~(size_t)15;  // slab from the aligned-down start
    p.sdn = (uint32_t)sdn;
    if ((size_t)p.rmax * (tpr / 32) * 24 > (size_t)K * sdn) return false;  // router partials
    p.o_dn = take((size_t)(K + 1) * sdn);
    const size_t up = (size_t)2 * p.upb;
    p.o_up = take(up);
    const size_t fb = (size_t)XL_SMEM + (size_t)11 * E * 4;
    if ((size_t)p.o_up + up - ((size_t)p.o_dn + sdn) < fb) {
        off = (size_t)p.o_dn + sdn + fb;
        off = (off + 127) & ~(size_t)127;
    }
    p.o_hb = take((size_t)p.upc * 4);
    p.o_part = take((size_t)std::max(8 * FD_WARPS, p.upc + 8) * 8);
    p.o_hst = take((size_t)FD_WARPS * FD_GROUP_BYTES);
    p.o_hq = take((size_t)(K + 1) * hslot_bytes(H));
    p.o_sel = take((size_t)2 * E * 4);
    p.o_ys = take((size_t)(K + 1) * rows_cap * (H / 128) * 4);
    p.o_res = take((size_t)rows_cap * 4);
    if (rows_cap > FD_THREADS) return false;  // residual rows: one thread each
    p.o_bar = take((size_t)(5 + K) * 8);
    p.total = (uint32_t)off;
    return p.total <= 227 * 1024;
}

int launch_decode_fused(const ofb_moe_config *cfg, const ofb_moe_weights *wt, const float *x, const float *resid,
                        float *out, uint32_t *idx_out, float *w_out, const FusedPlan &plan,
                        unsigned long long *cand, unsigned long long *hll, unsigned int *sync, int *stats,
                        cudaStream_t s) {
    FusedDecodeArgs a;
    a.W = wt->router; a.x = x; a.gate_v = wt->shexp_gate; a.resid = resid; a.out = out;
    a.gate = (const uint8_t *)wt->gate_exps; a.up = (const uint8_t *)wt->up_exps;
    a.down = (const uint8_t *)wt->down_exps;
    a.gate_sh = (const uint8_t *)wt->gate_shexp; a.up_sh = (const uint8_t *)wt->up_shexp;
    a.down_sh = (const uint8_t *)wt->down_shexp;
    a.D = cfg->d_model; a.H = cfg->hidden; a.E = cfg->n_experts; a.K = cfg->top_k;
    a.routing = cfg->routing; a.renorm = cfg->renorm;
    a.has_shared = wt->gate_shexp && wt->up_shexp && wt->down_shexp;
    a.use_gate = a.has_shared && cfg->shared_gate && wt->shexp_gate;
    const double u = 0x1.0p-24, n = (double)cfg->d_model;
    a.bound_scale = (1.0 + 0x1.0p-9) * u;
    a.ngam = n * (n * u / (1.0 - n * u));
    a.cand = cand; a.hll = hll; a.sync = sync;
    a.idx_out = idx_out; a.w_out = w_out; a.stats = stats;
    a.p = plan;
    static size_t attr[64];
    cudaError_t e = ensure_dyn_smem(decode_fused_kernel, plan.total, attr);
    if (e != cudaSuccess) return cuda_status(e, "decode_fused smem attribute");
    e = launch_pdl(decode_fused_kernel, dim3(plan.G), dim3(FD_THREADS), plan.total, s, a);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "decode_fused launch");
}

}  // namespace ofb
