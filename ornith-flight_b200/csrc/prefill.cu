// prefill.cu — grouped expert GEMMs on the 5th-generation tensor cores
// (tcgen05 + TMEM) for prefill-sized batches.
//
// Per expert e with n_e routed tokens (CSR slot from the dispatch plan), the
// layer is two GEMMs:
//   up:   H_e[n_e x 512]  = silu(X_e G_e^T) * (X_e U_e^T),  K = 2048
//   down: Y_e[n_e x 2048] = H_e Dn_e^T,                     K = 512
// both computed transposed, D = A . B^T with A = dequantised weight rows
// (M = 128 rows per CTA) and B = token rows (N <= 256 per tile), so the
// ragged token dimension is the MMA's N and every CTA tile is a full 128-row
// weight block.
//  * A: each thread owns one weight row; the raw Q4_K / Q6_K bytes for the
//    next 64-element K slice are loaded into registers while the tensor core
//    works on the current one, then dequantised (the reference's exact fp32
//    value, rounded to bf16) straight into shared memory in the canonical
//    no-swizzle K-major layout (8x16-byte core matrices).
//  * B: token rows are gathered from a bf16 copy of x (16.8 MB at 4096
//    tokens: L2-resident) or from the bf16 h of phase 1, 32 bytes per load.
//  * one elected thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32)
//    into TMEM; tcgen05.commit arrives on a per-stage mbarrier, which is what
//    frees the stage for refilling (two stages in flight).
//  * epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//    32w..32w+31 = its 32 weight rows); up writes h = silu(g)*u as bf16 in
//    slot order, down adds w * y into out with fp32 reductions.
// Every mbarrier wait is bounded: on timeout the kernel records an error
// flag, releases its TMEM and returns (the host reports OFB_ECUDA).
#include "common.cuh"
#include "moe.cuh"

namespace ofb {

constexpr int PF_M = 128;        // weight rows per CTA (MMA M)
constexpr int PF_NMAX = 256;     // token rows per tile (MMA N, max)
constexpr int PF_KS = 64;        // K elements per pipeline stage
constexpr int PF_THREADS = 128;
constexpr int A_LBO = (PF_M / 8) * 128;        // 2048 B between 8-element K chunks
constexpr int B_LBO = (PF_NMAX / 8) * 128;     // 4096 B
constexpr int A_STAGE = 8 * A_LBO;             // 16 KB
constexpr int B_STAGE = 8 * B_LBO;             // 32 KB
constexpr long long WAIT_LIMIT = 1ll << 26;    // try_wait polls before giving up

struct PrefillArgs {
    int T, D, H, E, K;
    int shared_gate;
    const uint8_t *gate, *up, *down, *gate_sh, *up_sh, *down_sh;
    const int *slot_expert, *slot_start, *assign;
    const int *n_tiles, *tile_slot, *tile_start, *tile_n;
    const __nv_bfloat16 *xb;  // [T][D]
    __nv_bfloat16 *hb;        // [A][H], slot order
    const float *w, *gsc;
    float *out;
    int *err;
};

// ---- PTX helpers ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
// Bounded wait for the mbarrier phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity) {
    const uint32_t a = smem_u32(b);
    for (long long i = 0; i < WAIT_LIMIT; i++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.b32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
           ((uint64_t)(sbo >> 4) << 32) | (1ull << 46);
}
// bf16 x bf16 -> f32, both K-major, M = 128.
__device__ __forceinline__ uint32_t instr_desc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(PF_M >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
        smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void async_proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t tmem_alloc(uint32_t *slot, uint32_t ncols) {
    if ((threadIdx.x >> 5) == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return *slot;
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if ((threadIdx.x >> 5) == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&p);
}

// smem byte offset of (row, 8-element K chunk) in a no-swizzle K-major tile
__device__ __forceinline__ uint32_t core_off(int row, int chunk, int lbo) {
    return chunk * lbo + (row >> 3) * 128 + (row & 7) * 16;
}

// ---- B operand: token rows ---------------------------------------------------
// 256 rows x 64 K of bf16 = 1024 units of 32 bytes; thread t owns units
// t + 128 j (j < 8): row = 8 g + r, chunk pair cp (chunks 2cp, 2cp+1).
struct BRegs { uint4 v[8][2]; };

__device__ __forceinline__ void b_load(BRegs &br, const __nv_bfloat16 *const *rowp, int n_rows, int k0) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int u = threadIdx.x + PF_THREADS * j;
        const int r = u & 7, cp = (u >> 3) & 3, g = u >> 5;
        const int row = g * 8 + r;
        if (row < n_rows) {
            const uint4 *src = reinterpret_cast<const uint4 *>(rowp[row] + k0 + cp * 16);
            br.v[j][0] = __ldg(src);
            br.v[j][1] = __ldg(src + 1);
        } else {
            br.v[j][0] = br.v[j][1] = make_uint4(0, 0, 0, 0);
        }
    }
}
__device__ __forceinline__ void b_store(const BRegs &br, uint8_t *sb) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int u = threadIdx.x + PF_THREADS * j;
        const int r = u & 7, cp = (u >> 3) & 3, g = u >> 5;
        const int row = g * 8 + r;
        *reinterpret_cast<uint4 *>(sb + core_off(row, 2 * cp, B_LBO)) = br.v[j][0];
        *reinterpret_cast<uint4 *>(sb + core_off(row, 2 * cp + 1, B_LBO)) = br.v[j][1];
    }
}

// ---- A operand, Q4_K: row slice [k0, k0+64) = chunk c of block b -----------
struct Q4Regs { uint4 hdr, qa, qb; };
__device__ __forceinline__ void q4_load(Q4Regs &q, const uint8_t *row, int stage) {
    const uint8_t *blk = row + (stage >> 2) * Q4K_BYTES;
    const int c = stage & 3;
    q.hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    q.qa = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + c * 32));
    q.qb = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + c * 32));
}
__device__ __forceinline__ void q4_store(const Q4Regs &q, int stage, uint8_t *sa) {
    const int c = stage & 3, r = threadIdx.x;
    const uint32_t s[3] = {q.hdr.y, q.hdr.z, q.hdr.w};
    int sc0, m0, sc1, m1;
    q4k_scale_min(s, 2 * c, sc0, m0);
    q4k_scale_min(s, 2 * c + 1, sc1, m1);
    const float d = half_bits_ref(q.hdr.x & 0xFFFFu), dmin = half_bits_ref(q.hdr.x >> 16);
    const float d0 = __fmul_rn(d, (float)sc0), mm0 = __fmul_rn(dmin, (float)m0);
    const float d1 = __fmul_rn(d, (float)sc1), mm1 = __fmul_rn(dmin, (float)m1);
    const uint32_t qw[8] = {q.qa.x, q.qa.y, q.qa.z, q.qa.w, q.qb.x, q.qb.y, q.qb.z, q.qb.w};
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
        // chunks 0-3: low nibbles of bytes 8ch..8ch+7; chunks 4-7: high nibbles
        const int wb = (ch & 3) * 2;
        const bool hi = ch >= 4;
        const float dd = hi ? d1 : d0, mm = hi ? mm1 : mm0;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t byte = (qw[wb + (i >> 2)] >> (8 * (i & 3))) & 0xFFu;
            v[i] = q4k_value(dd, mm, hi ? (int)(byte >> 4) : (int)(byte & 0xF));
        }
        *reinterpret_cast<uint4 *>(sa + core_off(r, ch, A_LBO)) =
            make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                       pack_bf16(v[6], v[7]));
    }
}

// ---- A operand, Q6_K: row slice [k0, k0+64) ----------------------------------
// 64-element chunk q of a block: half = q/2, quads 2*(q%2) and 2*(q%2)+1.
struct Q6Regs { uint16_t ql[32], qh[16], sc[2], d; };
__device__ __forceinline__ void q6_load(Q6Regs &q, const uint8_t *row, int stage) {
    const uint8_t *blk = row + (stage >> 2) * Q6K_BYTES;
    const int c = stage & 3, half = c >> 1;
    const uint16_t *ql = reinterpret_cast<const uint16_t *>(blk + half * 64);
    const uint16_t *qh = reinterpret_cast<const uint16_t *>(blk + 128 + half * 32);
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(blk + 192 + half * 8 + (c & 1) * 4);
#pragma unroll
    for (int i = 0; i < 32; i++) q.ql[i] = __ldg(ql + i);
#pragma unroll
    for (int i = 0; i < 16; i++) q.qh[i] = __ldg(qh + i);
    q.sc[0] = __ldg(sc);
    q.sc[1] = __ldg(sc + 1);
    q.d = __ldg(reinterpret_cast<const uint16_t *>(blk + 208));
}
__device__ __forceinline__ void q6_store(const Q6Regs &q, int stage, uint8_t *sa) {
    const int c = stage & 3, r = threadIdx.x, pair = c & 1;
    const float d = half_bits_ref(q.d);
    // scales for (quad 2*pair, is 0/1) and (quad 2*pair+1, is 0/1)
    const int8_t s00 = (int8_t)(q.sc[0] & 0xFF), s01 = (int8_t)(q.sc[0] >> 8);
    const int8_t s10 = (int8_t)(q.sc[1] & 0xFF), s11 = (int8_t)(q.sc[1] >> 8);
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
        // element kk = 8ch + i: quad = 2*pair + kk/32, l = kk % 32
        const int qsel = ch >> 2;          // 0: first quad of the pair, 1: second
        const int quad = 2 * pair + qsel;
        const int l0 = (ch & 3) * 8;
        const int8_t scv = qsel ? ((l0 >> 4) ? s11 : s10) : ((l0 >> 4) ? s01 : s00);
        const float ds = __fmul_rn(d, (float)scv);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int l = l0 + i;
            const int qlidx = ((quad & 1) ? 32 : 0) + l;
            const uint32_t lb = (q.ql[qlidx >> 1] >> (8 * (qlidx & 1))) & 0xFF;
            const int nib = (quad < 2) ? (int)(lb & 0xF) : (int)(lb >> 4);
            const uint32_t hb = (q.qh[l >> 1] >> (8 * (l & 1))) & 0xFF;
            const int top = (hb >> (2 * quad)) & 3;
            v[i] = __fmul_rn(ds, (float)((nib | (top << 4)) - 32));
        }
        *reinterpret_cast<uint4 *>(sa + core_off(r, ch, A_LBO)) =
            make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                       pack_bf16(v[6], v[7]));
    }
}

__device__ __forceinline__ int asg_token_p(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

// ---- phase 1: gate/up ----------------------------------------------------------
// grid (max_tiles, H/128); dynamic smem: 2 stages x (Ag, Au, B) + bookkeeping.
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_up_kernel(PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t psm[];
    __shared__ uint64_t bars[2];
    __shared__ uint32_t tslot;
    __shared__ const __nv_bfloat16 *rowp[PF_NMAX];
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int u = a.tile_slot[tile], s0 = a.tile_start[tile], n = a.tile_n[tile];
    const int e = a.slot_expert[u];
    const int m0 = blockIdx.y * PF_M;
    const int TK = a.T * a.K;
    const int nbr = a.D / QK;
    const size_t row_bytes = (size_t)nbr * Q4K_BYTES, exp_bytes = row_bytes * a.H;
    const uint8_t *grow = (e == a.E ? a.gate_sh : a.gate + e * exp_bytes) + (m0 + threadIdx.x) * row_bytes;
    const uint8_t *urow = (e == a.E ? a.up_sh : a.up + e * exp_bytes) + (m0 + threadIdx.x) * row_bytes;
    for (int i = threadIdx.x; i < PF_NMAX; i += PF_THREADS)
        rowp[i] = a.xb + (size_t)(i < n ? asg_token_p(a.assign[s0 + i], TK, a.K) : 0) * a.D;
    if (threadIdx.x == 0) { mbar_init(&bars[0], 1); mbar_init(&bars[1], 1); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 512);  // gate: cols [0,256), up: [256,512)

    const int nn = (n + 15) & ~15;  // MMA N: multiple of 16
    const uint32_t idesc = instr_desc(nn);
    const int nstages = a.D / PF_KS;
    Q4Regs gq, uq;
    BRegs br;
    q4_load(gq, grow, 0);
    q4_load(uq, urow, 0);
    b_load(br, rowp, n, 0);
    bool ok = true;
    for (int i = 0; i < nstages; i++) {
        const int s = i & 1;
        uint8_t *sg = psm + s * (2 * A_STAGE + B_STAGE), *su = sg + A_STAGE, *sb = sg + 2 * A_STAGE;
        if (i >= 2) ok = ok && mbar_wait(&bars[s], ((i - 2) >> 1) & 1);
        q4_store(gq, i, sg);
        q4_store(uq, i, su);
        b_store(br, sb);
        if (i + 1 < nstages) {
            q4_load(gq, grow, i + 1);
            q4_load(uq, urow, i + 1);
            b_load(br, rowp, n, (i + 1) * PF_KS);
        }
        async_proxy_fence();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t ag = smem_u32(sg), au = smem_u32(su), bb = smem_u32(sb);
#pragma unroll
            for (int kk = 0; kk < PF_KS / 16; kk++) {
                const uint64_t bd = smem_desc(bb + kk * 2 * B_LBO, B_LBO, 128);
                mma_bf16(tbase, smem_desc(ag + kk * 2 * A_LBO, A_LBO, 128), bd, idesc, (i | kk) != 0);
                mma_bf16(tbase + 256, smem_desc(au + kk * 2 * A_LBO, A_LBO, 128), bd, idesc, (i | kk) != 0);
            }
            mma_commit(&bars[s]);
        }
    }
    ok = ok && mbar_wait(&bars[(nstages - 1) & 1], ((nstages - 1) >> 1) & 1);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else {
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int m = m0 + w * 32 + lane;
        const uint32_t lane_off = (uint32_t)(w * 32) << 16;
        for (int j0 = 0; j0 < nn; j0 += 8) {
            float g[8], uu[8];
            tmem_ld8(tbase + lane_off + j0, g);
            tmem_ld8(tbase + lane_off + 256 + j0, uu);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j0 + j >= n) break;
                const float gv = g[j];
                const float sl = gv < -50.f ? 0.f : (gv > 50.f ? gv : gv / (1.f + expf(-gv)));
                a.hb[(size_t)(s0 + j0 + j) * a.H + m] = __float2bfloat16_rn(sl * uu[j]);
            }
        }
    }
    tmem_free(tbase, 512);
}

// ---- phase 2: down + weighted combine -----------------------------------------
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_down_kernel(PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t psm[];
    __shared__ uint64_t bars[2];
    __shared__ uint32_t tslot;
    __shared__ const __nv_bfloat16 *rowp[PF_NMAX];
    __shared__ int tok[PF_NMAX];
    __shared__ float wgt[PF_NMAX];
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int u = a.tile_slot[tile], s0 = a.tile_start[tile], n = a.tile_n[tile];
    const int e = a.slot_expert[u];
    const int n0 = blockIdx.y * PF_M;
    const int TK = a.T * a.K;
    const int nbk = a.H / QK;
    const size_t row_bytes = (size_t)nbk * Q6K_BYTES, exp_bytes = row_bytes * a.D;
    const uint8_t *drow = (e == a.E ? a.down_sh : a.down + e * exp_bytes) + (n0 + threadIdx.x) * row_bytes;
    for (int i = threadIdx.x; i < PF_NMAX; i += PF_THREADS) {
        rowp[i] = a.hb + (size_t)(s0 + (i < n ? i : 0)) * a.H;
        if (i < n) {
            const int asg = a.assign[s0 + i];
            const int t = asg_token_p(asg, TK, a.K);
            tok[i] = t;
            wgt[i] = asg < TK ? a.w[asg] : (a.shared_gate ? a.gsc[t] : 1.0f);
        }
    }
    if (threadIdx.x == 0) { mbar_init(&bars[0], 1); mbar_init(&bars[1], 1); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 256);

    const int nn = (n + 15) & ~15;
    const uint32_t idesc = instr_desc(nn);
    const int nstages = a.H / PF_KS;
    Q6Regs dq;
    BRegs br;
    q6_load(dq, drow, 0);
    b_load(br, rowp, n, 0);
    bool ok = true;
    for (int i = 0; i < nstages; i++) {
        const int s = i & 1;
        uint8_t *sa = psm + s * (A_STAGE + B_STAGE), *sb = sa + A_STAGE;
        if (i >= 2) ok = ok && mbar_wait(&bars[s], ((i - 2) >> 1) & 1);
        q6_store(dq, i, sa);
        b_store(br, sb);
        if (i + 1 < nstages) {
            q6_load(dq, drow, i + 1);
            b_load(br, rowp, n, (i + 1) * PF_KS);
        }
        async_proxy_fence();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t aa = smem_u32(sa), bb = smem_u32(sb);
#pragma unroll
            for (int kk = 0; kk < PF_KS / 16; kk++)
                mma_bf16(tbase, smem_desc(aa + kk * 2 * A_LBO, A_LBO, 128),
                         smem_desc(bb + kk * 2 * B_LBO, B_LBO, 128), idesc, (i | kk) != 0);
            mma_commit(&bars[s]);
        }
    }
    ok = ok && mbar_wait(&bars[(nstages - 1) & 1], ((nstages - 1) >> 1) & 1);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else {
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int row = n0 + w * 32 + lane;
        const uint32_t lane_off = (uint32_t)(w * 32) << 16;
        for (int j0 = 0; j0 < nn; j0 += 8) {
            float y[8];
            tmem_ld8(tbase + lane_off + j0, y);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j0 + j >= n) break;
                atomicAdd(a.out + (size_t)tok[j0 + j] * a.D + row, wgt[j0 + j] * y[j]);
            }
        }
    }
    tmem_free(tbase, 256);
}

// ---- helpers: x to bf16, tile list ---------------------------------------------
__global__ void to_bf16_kernel(const float *__restrict__ x, size_t n, __nv_bfloat16 *__restrict__ y) {
    for (size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 4; i < n;
         i += (size_t)gridDim.x * blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(x + i);
        uint2 o = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
        *reinterpret_cast<uint2 *>(y + i) = o;
    }
}

// One block: split every slot into tiles of at most 256 tokens.
__global__ void tile_plan_kernel(const int *n_slots, const int *slot_start, int *n_tiles, int *tile_slot,
                                 int *tile_start, int *tile_n) {
    __shared__ int base[1025];
    const int ns = *n_slots;
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int u = 0; u < ns; u++) {
            base[u] = acc;
            acc += (slot_start[u + 1] - slot_start[u] + PF_NMAX - 1) / PF_NMAX;
        }
        base[ns] = acc;
        *n_tiles = acc;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < ns; u += blockDim.x) {
        const int st = slot_start[u], cnt = slot_start[u + 1] - st;
        for (int k = 0; k < base[u + 1] - base[u]; k++) {
            const int t = base[u] + k;
            tile_slot[t] = u;
            tile_start[t] = st + k * PF_NMAX;
            tile_n[t] = min(PF_NMAX, cnt - k * PF_NMAX);
        }
    }
}

int prefill_max_tiles(int T, int K, int E) {
    const int assignments = T * K + T;
    const int slots = (T * K < E ? T * K : E) + 1;
    return assignments / PF_NMAX + slots + 1;
}

bool prefill_supported(int D, int H) { return D % 256 == 0 && H % 256 == 0 && H % PF_M == 0 && D % PF_M == 0; }

int launch_prefill(const LayerArgs &la, const float *x, int *n_slots, __nv_bfloat16 *xb, __nv_bfloat16 *hb,
                   int *tiles, int *err, cudaStream_t s) {
    const int T = la.T, D = la.D, H = la.H;
    const int max_tiles = prefill_max_tiles(T, la.K, la.E);
    int *n_tiles = tiles, *tile_slot = tiles + 1, *tile_start = tile_slot + max_tiles,
        *tile_n = tile_start + max_tiles;
    to_bf16_kernel<<<grid_for((size_t)T * D / 4, 256, 148 * 8), 256, 0, s>>>(x, (size_t)T * D, xb);
    tile_plan_kernel<<<1, 256, 0, s>>>(n_slots, la.slot_start, n_tiles, tile_slot, tile_start, tile_n);
    PrefillArgs a;
    a.T = T; a.D = D; a.H = H; a.E = la.E; a.K = la.K;
    a.shared_gate = la.shared_gate;
    a.gate = la.gate; a.up = la.up; a.down = la.down;
    a.gate_sh = la.gate_sh; a.up_sh = la.up_sh; a.down_sh = la.down_sh;
    a.slot_expert = la.slot_expert; a.slot_start = la.slot_start; a.assign = la.assign;
    a.n_tiles = n_tiles; a.tile_slot = tile_slot; a.tile_start = tile_start; a.tile_n = tile_n;
    a.xb = xb; a.hb = hb; a.w = la.w; a.gsc = la.gsc; a.out = la.out; a.err = err;
    const int smem_up = 2 * (2 * A_STAGE + B_STAGE);
    const int smem_dn = 2 * (A_STAGE + B_STAGE);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prefill_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_up);
        cudaFuncSetAttribute(prefill_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dn);
        attr = true;
    }
    // out starts as the residual (or zero); the down kernel adds w * y into it
    cudaError_t e;
    if (!la.resid) e = cudaMemsetAsync(la.out, 0, (size_t)T * D * sizeof(float), s);
    else if (la.resid != la.out)
        e = cudaMemcpyAsync(la.out, la.resid, (size_t)T * D * sizeof(float), cudaMemcpyDeviceToDevice, s);
    else e = cudaSuccess;
    if (e != cudaSuccess) return cuda_status(e, "prefill out init");
    prefill_up_kernel<<<dim3(max_tiles, H / PF_M), PF_THREADS, smem_up, s>>>(a);
    prefill_down_kernel<<<dim3(max_tiles, D / PF_M), PF_THREADS, smem_dn, s>>>(a);
    OFB_CHECK_LAUNCH("prefill kernels");
    return OFB_OK;
}

}  // namespace ofb
