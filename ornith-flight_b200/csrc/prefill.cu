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

// ---- async copies -----------------------------------------------------------
// 16-byte global->shared copy; src_bytes = 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// One TMA bulk copy global -> shared completing on an mbarrier (no multicast).
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 4 bytes at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_u32_2b(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(b[0], b[1], (unsigned)(a & 3) * 8);
}

// byte k of w as a float (exact small integer): 2^23 + byte, minus 2^23 + bias
template <int K>
__device__ __forceinline__ float byte_f(uint32_t w, float bias) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + K)) - bias;
}

constexpr int PF_NT = 256;                    // threads per CTA (8 warps)
constexpr int PF_STG = 3;                     // cp.async pipeline depth
constexpr int B_LBO_P = B_LBO + 16;           // padded: the 8 chunks of a row hit 8 bank groups
constexpr int B_STAGE_P = 8 * B_LBO_P;
constexpr int RAW4 = PF_M * 48;               // raw Q4_K bytes of one matrix per stage

// B: 2048 16-byte copies per stage; thread t copies j = t + 256 k (k < 8):
// chunk = j & 7, row = j >> 3 (a quarter-warp copies one 128-byte row).
// The per-thread sources and destinations are fixed for the whole K loop.
struct BPlan { const __nv_bfloat16 *src[8]; uint32_t dst[8]; uint32_t bytes[8]; };
__device__ __forceinline__ void b_plan(BPlan &p, const __nv_bfloat16 *const *rowp, int n_rows) {
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int j = threadIdx.x + PF_NT * k;
        const int ch = j & 7, row = j >> 3;
        const bool ok = row < n_rows;
        p.src[k] = rowp[ok ? row : 0] + ch * 8;
        p.dst[k] = core_off(row, ch, B_LBO_P);
        p.bytes[k] = ok ? 16u : 0u;
    }
}
__device__ __forceinline__ void b_issue(const BPlan &p, uint32_t sb, int k0) {
#pragma unroll
    for (int k = 0; k < 8; k++) cp_async16(sb + p.dst[k], p.src[k] + k0, p.bytes[k]);
}

// Q4_K raw bytes of one stage (16 B header + 32 quant bytes per row, both
// matrices): 768 copies, thread t copies t, t+256, t+512.
struct QPlan { const uint8_t *src[3]; uint32_t dst[3]; int part[3]; };
__device__ __forceinline__ void q4_plan(QPlan &p, const uint8_t *g0, const uint8_t *u0, size_t row_bytes) {
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const int j = threadIdx.x + PF_NT * k;
        const int mat = j / 384, rem = j - mat * 384, row = rem / 3, part = rem - row * 3;
        p.src[k] = (mat ? u0 : g0) + row * row_bytes;
        p.dst[k] = mat * RAW4 + row * 48 + part * 16;
        p.part[k] = part;
    }
}
__device__ __forceinline__ void q4_issue(const QPlan &p, uint32_t sraw, int stage) {
    const int b = stage >> 2, c = stage & 3;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const int off = b * Q4K_BYTES + (p.part[k] ? 16 + c * 32 + (p.part[k] - 1) * 16 : 0);
        cp_async16(sraw + p.dst[k], p.src[k] + off, 16u);
    }
}

// Paired fp32 arithmetic (sm_100a f32x2): two lanes of work per instruction.
__device__ __forceinline__ unsigned long long f2pack(float a, float b) {
    unsigned long long p;
    asm("mov.b64 %0, {%1,%2};" : "=l"(p) : "f"(a), "f"(b));
    return p;
}
__device__ __forceinline__ uint32_t f2_fma_bf16(unsigned long long x, unsigned long long m,
                                                 unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(m), "l"(c));
    float lo, hi;
    asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
    return pack_bf16(lo, hi);
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// two bytes (k, k+1) of w as exact floats 2^23 + byte, as a pair
template <int K>
__device__ __forceinline__ unsigned long long byte_pair(uint32_t w) {
    return f2pack(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + K)),
                  __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541u + K)));
}

// Dequantise one matrix's stage: thread (row r, half hh) writes chunks
// 4hh..4hh+3 (low nibbles for hh = 0, high for hh = 1). Value = (d*sc)*q -
// dmin*m as one fused multiply-add: d*sc*q is exact in fp32 (<= 21 bits), so
// the result equals the reference's two separately rounded operations.
__device__ __forceinline__ void q4_deq(const uint8_t *raw, int stage, uint8_t *sa) {
    const int r = threadIdx.x & (PF_M - 1), hh = threadIdx.x >> 7, c = stage & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * 48);
    const uint4 qa = *reinterpret_cast<const uint4 *>(raw + r * 48 + 16);
    const uint4 qb = *reinterpret_cast<const uint4 *>(raw + r * 48 + 32);
    const uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    int sc, mn;
    q4k_scale_min(s, 2 * c + hh, sc, mn);
    const float dd = __fmul_rn(half_bits_ref(hdr.x & 0xFFFFu), (float)sc);
    const float mm = __fmul_rn(half_bits_ref(hdr.x >> 16), (float)mn);
    const unsigned long long d2 = f2pack(dd, dd), nm2 = f2pack(-mm, -mm);
    const unsigned long long nb2 = f2pack(-8388608.0f, -8388608.0f);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int sh = 4 * hh;
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const uint32_t w0 = (qw[2 * ch] >> sh) & 0x0F0F0F0Fu, w1 = (qw[2 * ch + 1] >> sh) & 0x0F0F0F0Fu;
        // q as exact floats, then one paired FMA per two elements
        const uint32_t p0 = f2_fma_bf16(f2_add(byte_pair<0>(w0), nb2), d2, nm2);
        const uint32_t p1 = f2_fma_bf16(f2_add(byte_pair<2>(w0), nb2), d2, nm2);
        const uint32_t p2 = f2_fma_bf16(f2_add(byte_pair<0>(w1), nb2), d2, nm2);
        const uint32_t p3 = f2_fma_bf16(f2_add(byte_pair<2>(w1), nb2), d2, nm2);
        *reinterpret_cast<uint4 *>(sa + core_off(r, 4 * hh + ch, A_LBO)) = make_uint4(p0, p1, p2, p3);
    }
}

// Q6_K stage from the raw slab in shared memory: thread (row r, hh) writes the
// 32 elements of quad 2*(chunk%2)+hh. Value = (d*sc)*(q-32), one rounding.
__device__ __forceinline__ void q6_deq(const uint8_t *slab, int row_bytes, int stage, uint8_t *sa) {
    const int r = threadIdx.x & (PF_M - 1), hh = threadIdx.x >> 7;
    const int b = stage >> 2, q64 = stage & 3, half6 = q64 >> 1, quad = 2 * (q64 & 1) + hh;
    const uint8_t *blk = slab + r * row_bytes + b * Q6K_BYTES;
    const uint8_t *ql = blk + half6 * 64 + (quad & 1) * 32;
    const uint8_t *qh = blk + 128 + half6 * 32;
    const uint32_t scw = (uint32_t)blk[192 + half6 * 8 + quad * 2] | ((uint32_t)blk[193 + half6 * 8 + quad * 2] << 8);
    const float d = half_bits_ref((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
    const float ds0 = __fmul_rn(d, (float)(int8_t)(scw & 0xFF)), ds1 = __fmul_rn(d, (float)(int8_t)(scw >> 8));
    const float bias = 8388608.0f + 32.0f;
    const int nsh = (quad >= 2) ? 4 : 0, hsh = 2 * quad;
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const float ds = ch < 2 ? ds0 : ds1;  // l = 8ch..8ch+7, is = l/16
        uint32_t q[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
            const uint32_t wl = lds_u32_2b(ql + ch * 8 + h2 * 4), wh = lds_u32_2b(qh + ch * 8 + h2 * 4);
            q[h2] = ((wl >> nsh) & 0x0F0F0F0Fu) | (((wh >> hsh) & 0x03030303u) << 4);
        }
        const float v0 = __fmul_rn(ds, byte_f<0>(q[0], bias)), v1 = __fmul_rn(ds, byte_f<1>(q[0], bias));
        const float v2 = __fmul_rn(ds, byte_f<2>(q[0], bias)), v3 = __fmul_rn(ds, byte_f<3>(q[0], bias));
        const float v4 = __fmul_rn(ds, byte_f<0>(q[1], bias)), v5 = __fmul_rn(ds, byte_f<1>(q[1], bias));
        const float v6 = __fmul_rn(ds, byte_f<2>(q[1], bias)), v7 = __fmul_rn(ds, byte_f<3>(q[1], bias));
        *reinterpret_cast<uint4 *>(sa + core_off(r, 4 * hh + ch, A_LBO)) =
            make_uint4(pack_bf16(v0, v1), pack_bf16(v2, v3), pack_bf16(v4, v5), pack_bf16(v6, v7));
    }
}

__device__ __forceinline__ int asg_token_p(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

// ---- phase 1: gate/up ----------------------------------------------------------
// Iteration i: (1) stage i's copies have landed; (2) dequantise it into the
// bf16 A buffer i%2 (free: MMA i-2 was waited for in iteration i-1) while the
// tensor core runs MMA i-1; (3) issue MMA i; (4) wait for MMA i-1, whose B
// buffer is the one stage i+2 refills, then issue stage i+2's copies.
constexpr int UP_SMEM = PF_STG * (2 * RAW4 + B_STAGE_P) + 2 * (2 * A_STAGE);

__global__ void __launch_bounds__(PF_NT, 1) prefill_up_kernel(PrefillArgs a) {
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
    const size_t row_bytes = (size_t)(a.D / QK) * Q4K_BYTES, exp_bytes = row_bytes * a.H;
    const uint8_t *g0 = (e == a.E ? a.gate_sh : a.gate + e * exp_bytes) + (size_t)m0 * row_bytes;
    const uint8_t *u0 = (e == a.E ? a.up_sh : a.up + e * exp_bytes) + (size_t)m0 * row_bytes;
    for (int i = threadIdx.x; i < PF_NMAX; i += PF_NT)
        rowp[i] = a.xb + (size_t)(i < n ? asg_token_p(a.assign[s0 + i], TK, a.K) : 0) * a.D;
    if (threadIdx.x == 0) { mbar_init(&bars[0], 1); mbar_init(&bars[1], 1); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 512);  // gate: cols [0,256), up: [256,512)

    uint8_t *raw = psm;                                   // [PF_STG][2*RAW4]
    uint8_t *bst = psm + PF_STG * 2 * RAW4;               // [PF_STG][B_STAGE_P]
    uint8_t *abf = bst + PF_STG * B_STAGE_P;              // [2][gate A | up A]
    const int nn = (n + 15) & ~15;
    const uint32_t idesc = instr_desc(nn);
    const int nstages = a.D / PF_KS;
    __syncthreads();  // rowp
    BPlan bp;
    b_plan(bp, rowp, n);
    QPlan qp;
    q4_plan(qp, g0, u0, row_bytes);
    for (int i = 0; i < PF_STG - 1; i++) {
        if (i < nstages) {
            q4_issue(qp, smem_u32(raw + i * 2 * RAW4), i);
            b_issue(bp, smem_u32(bst + i * B_STAGE_P), i * PF_KS);
        }
        cp_async_commit();
    }
    bool ok = true;
    for (int i = 0; i < nstages; i++) {
        const int sr = i % PF_STG, sa = i & 1;
        cp_async_wait<PF_STG - 2>();
        __syncthreads();
        uint8_t *ag = abf + sa * 2 * A_STAGE, *au = ag + A_STAGE;
        q4_deq(raw + sr * 2 * RAW4, i, ag);
        q4_deq(raw + sr * 2 * RAW4 + RAW4, i, au);
        async_proxy_fence();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t ga = smem_u32(ag), ua = smem_u32(au), bb = smem_u32(bst + sr * B_STAGE_P);
#pragma unroll
            for (int kk = 0; kk < PF_KS / 16; kk++) {
                const uint64_t bd = smem_desc(bb + kk * 2 * B_LBO_P, B_LBO_P, 128);
                mma_bf16(tbase, smem_desc(ga + kk * 2 * A_LBO, A_LBO, 128), bd, idesc, (i | kk) != 0);
                mma_bf16(tbase + 256, smem_desc(ua + kk * 2 * A_LBO, A_LBO, 128), bd, idesc, (i | kk) != 0);
            }
            mma_commit(&bars[sa]);
        }
        // one warp waits for MMA i-1 (its B buffer is refilled next); the
        // others wait at the barrier instead of polling
        if (i >= 1) {
            if (threadIdx.x < 32) ok = ok && mbar_wait(&bars[(i - 1) & 1], ((i - 1) >> 1) & 1);
            __syncthreads();
        }
        const int nx = i + PF_STG - 1;
        if (nx < nstages) {
            q4_issue(qp, smem_u32(raw + (nx % PF_STG) * 2 * RAW4), nx);
            b_issue(bp, smem_u32(bst + (nx % PF_STG) * B_STAGE_P), nx * PF_KS);
        }
        cp_async_commit();
    }
    if (threadIdx.x < 32) ok = ok && mbar_wait(&bars[(nstages - 1) & 1], ((nstages - 1) >> 1) & 1);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else {
        // warp w reads TMEM lanes 32*(w%4).. (its rows), columns of half w/4
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, q = w & 3;
        const int m = m0 + q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int half = nn / 2, j_beg = (w >> 2) * half;
        for (int j0 = j_beg; j0 < j_beg + half; j0 += 8) {
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
// The CTA's 128 Q6_K rows are one contiguous, 16-byte aligned slab
// (128 x 420 B): one TMA bulk copy brings it in; stages then only copy B.
__host__ __device__ inline int down_slab_bytes(int H) { return PF_M * (H / QK) * Q6K_BYTES; }
__host__ __device__ inline int down_smem(int H) {
    return down_slab_bytes(H) + 16 + PF_STG * B_STAGE_P + 2 * A_STAGE;
}

__global__ void __launch_bounds__(PF_NT, 1) prefill_down_kernel(PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t psm[];
    __shared__ uint64_t bars[3];
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
    const int row_bytes = (a.H / QK) * Q6K_BYTES;
    const size_t exp_bytes = (size_t)row_bytes * a.D;
    const uint8_t *slab_src = (e == a.E ? a.down_sh : a.down + e * exp_bytes) + (size_t)n0 * row_bytes;
    uint8_t *bst = psm;                                    // [PF_STG][B_STAGE_P]
    uint8_t *abf = bst + PF_STG * B_STAGE_P;               // [2][A_STAGE]
    uint8_t *slab = abf + 2 * A_STAGE;                     // raw Q6_K rows
    for (int i = threadIdx.x; i < PF_NMAX; i += PF_NT) {
        rowp[i] = a.hb + (size_t)(s0 + (i < n ? i : 0)) * a.H;
        if (i < n) {
            const int asg = a.assign[s0 + i];
            const int t = asg_token_p(asg, TK, a.K);
            tok[i] = t;
            wgt[i] = asg < TK ? a.w[asg] : (a.shared_gate ? a.gsc[t] : 1.0f);
        }
    }
    if (threadIdx.x == 0) { mbar_init(&bars[0], 1); mbar_init(&bars[1], 1); mbar_init(&bars[2], 1); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) bulk_copy(slab, slab_src, down_slab_bytes(a.H), &bars[2]);
    const uint32_t tbase = tmem_alloc(&tslot, 256);

    const int nn = (n + 15) & ~15;
    const uint32_t idesc = instr_desc(nn);
    const int nstages = a.H / PF_KS;
    BPlan bp;
    b_plan(bp, rowp, n);
    for (int i = 0; i < PF_STG - 1; i++) {
        if (i < nstages) b_issue(bp, smem_u32(bst + i * B_STAGE_P), i * PF_KS);
        cp_async_commit();
    }
    bool ok = mbar_wait(&bars[2], 0);
    for (int i = 0; i < nstages; i++) {
        const int sr = i % PF_STG, sa = i & 1;
        cp_async_wait<PF_STG - 2>();
        __syncthreads();
        uint8_t *ad = abf + sa * A_STAGE;
        q6_deq(slab, row_bytes, i, ad);
        async_proxy_fence();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t aa = smem_u32(ad), bb = smem_u32(bst + sr * B_STAGE_P);
#pragma unroll
            for (int kk = 0; kk < PF_KS / 16; kk++)
                mma_bf16(tbase, smem_desc(aa + kk * 2 * A_LBO, A_LBO, 128),
                         smem_desc(bb + kk * 2 * B_LBO_P, B_LBO_P, 128), idesc, (i | kk) != 0);
            mma_commit(&bars[sa]);
        }
        if (i >= 1) {
            if (threadIdx.x < 32) ok = ok && mbar_wait(&bars[(i - 1) & 1], ((i - 1) >> 1) & 1);
            __syncthreads();
        }
        const int nx = i + PF_STG - 1;
        if (nx < nstages) b_issue(bp, smem_u32(bst + (nx % PF_STG) * B_STAGE_P), nx * PF_KS);
        cp_async_commit();
    }
    if (threadIdx.x < 32) ok = ok && mbar_wait(&bars[(nstages - 1) & 1], ((nstages - 1) >> 1) & 1);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else {
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, q = w & 3;
        const int row = n0 + q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int half = nn / 2, j_beg = (w >> 2) * half;
        for (int j0 = j_beg; j0 < j_beg + half; j0 += 8) {
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
                   int *tiles, int *err, cudaStream_t s, cudaEvent_t before, cudaEvent_t between) {
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
    const int smem_up = UP_SMEM;
    const int smem_dn = down_smem(H);
    static int attr_dn = 0;
    if (!attr_dn) cudaFuncSetAttribute(prefill_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_up);
    if (smem_dn > attr_dn) {
        cudaFuncSetAttribute(prefill_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dn);
        attr_dn = smem_dn;
    }
    // out starts as the residual (or zero); the down kernel adds w * y into it
    cudaError_t e;
    if (!la.resid) e = cudaMemsetAsync(la.out, 0, (size_t)T * D * sizeof(float), s);
    else if (la.resid != la.out)
        e = cudaMemcpyAsync(la.out, la.resid, (size_t)T * D * sizeof(float), cudaMemcpyDeviceToDevice, s);
    else e = cudaSuccess;
    if (e != cudaSuccess) return cuda_status(e, "prefill out init");
    if (before) cudaEventRecord(before, s);
    prefill_up_kernel<<<dim3(max_tiles, H / PF_M), PF_NT, smem_up, s>>>(a);
    if (between) cudaEventRecord(between, s);
    prefill_down_kernel<<<dim3(max_tiles, D / PF_M), PF_NT, smem_dn, s>>>(a);
    OFB_CHECK_LAUNCH("prefill kernels");
    return OFB_OK;
}

}  // namespace ofb
