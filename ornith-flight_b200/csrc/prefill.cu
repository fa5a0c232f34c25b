// prefill.cu — grouped expert GEMMs on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for prefill-sized batches.
//
// Per expert e with n_e routed tokens (CSR slot from the dispatch plan), the
// layer is two GEMMs:
//   up:   H_e[n_e x H] = silu(X_e G_e^T) * (X_e U_e^T),  K = D
//   down: Y_e[n_e x D] = H_e Dn_e^T,                     K = H
// both computed transposed, D = A . B^T with A = dequantised weight rows
// (M = 128 rows per CTA) and B = token rows (N <= 256 per tile), so the
// ragged token dimension is the MMA's N and every CTA tile is a full 128-row
// weight block.
//  * B (token rows): TMA tile loads of 64 columns x 16 rows, as many as the
//    tile's rows need, per stage. A gather kernel first writes each
//    assignment's token row as bf16 in slot order (x rows for the up GEMM);
//    the up epilogue writes h in the same order, so every tile's B rows are
//    contiguous. 128-byte swizzled K-major layout, one mbarrier per stage.
//  * A (weights) lives in tensor memory: dequantising warps write their bf16
//    pairs straight from registers with tcgen05.st and the MMA reads A from
//    TMEM, so shared memory carries only B and the raw quant bytes. The raw
//    Q4_K bytes a stage needs (16-byte header and two 16-byte quant chunks of
//    each row's block) arrive by TMA through a 3D byte map (16-byte chunk x
//    chunk index x row); the Q6_K rows of a CTA are one contiguous, 16-byte
//    aligned slab (128 x 420 B) brought in by one bulk copy.
//  * TMEM columns: up = gate accumulator [0,192), up accumulator [192,384),
//    two A stages [384,512); down (persistent, two accumulators so that one
//    unit's epilogue overlaps the next unit's MMAs) = accumulators [0,192)
//    and [192,384), two A stages [384,448). Tiles hold at most 192 tokens
//    (the MMA's N).
//  * one thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32);
//    tcgen05.commit arrives on the mbarriers that free the stage's buffers.
//  * warp-specialised: warp 0 produces B, warp 2 raw A (TMA), warp 1 issues
//    the MMAs, warps 4..19 dequantise (warp w owns TMEM lanes 32*(w%4)..,
//    i.e. weight rows 32*(w%4).. of the CTA); the roles meet only on
//    full/empty mbarrier rings, so copies, dequantisation and tensor-core
//    work of different stages overlap.
//  * grid: (weight-row block, tile), so the CTAs sharing a tile's B rows run
//    next to each other and read them from L2.
//  * epilogue (warps 4..19): tcgen05.ld of the accumulator; up stages
//    h = silu(g)*u as bf16 in shared memory and stores whole 16-byte pieces
//    of each token's row, down adds w * y into out with fp32 reductions.
// Every TMA load here reads this GPU's own memory into this CTA only. Every mbarrier wait is bounded: on
// timeout the kernel records an error flag, releases its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "moe.cuh"

namespace ofb {

constexpr int PF_M = 128;        // weight rows per CTA (MMA M)
constexpr int PF_KS = 64;        // K elements per pipeline stage (= one 128-byte swizzle row)
constexpr int PF_DQ0 = 128;      // first dequantising thread
constexpr int PF_NDQW = 16;      // dequantising warps
constexpr int PF_STG = 4;        // ring depth for B
constexpr int PF_RAW = 3;        // raw Q4_K blocks in flight (108 KB of gate + up rows)
constexpr int PF_NA = 2;         // A stages in TMEM
constexpr int B_ROWS = 16;       // rows per B box
constexpr int B_STAGE = PF_NMAX * 128;     // 24 KB: up to 192 rows x 128 B
constexpr int RAW4 = PF_M * Q4K_BYTES;      // raw Q4_K bytes of one matrix per raw stage (one block)
constexpr long long WAIT_LIMIT = 1ll << 26;       // try_wait polls before giving up
constexpr unsigned long long WAIT_NS = 250000000;  // or this much time (0.25 s), whichever comes first

struct PrefillArgs {
    int T, D, H, E, K;
    int shared_gate;
    const uint8_t *gate, *up, *down, *gate_sh, *up_sh, *down_sh;
    const int *slot_expert, *slot_start, *assign;
    const int *n_tiles, *tile_slot, *tile_start, *tile_n;
    __nv_bfloat16 *hb;  // [A][H], slot order
    const float *w, *gsc;
    float *out;
    int *err;
};

// Optional per-CTA timing of the roles' waits (build with -DOFB_PF_TRACE):
// clock64 sums for the first 256 CTAs of each kernel, read back with
// ofb_debug_prefill_trace.
#ifdef OFB_PF_TRACE
__device__ unsigned long long g_pf_trace[2][256][32];
__device__ unsigned long long g_pf_span[2][8192][2];  // globaltimer start/end of every CTA
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned long long *pf_tr(int kern) {
    const int id = blockIdx.x + gridDim.x * blockIdx.y;
    if (threadIdx.x == 0 && id < 8192) g_pf_span[kern][id][0] = gtime();
    return id < 256 ? g_pf_trace[kern][id] : nullptr;
}
__device__ __forceinline__ void pf_end(int kern) {
    const int id = blockIdx.x + gridDim.x * blockIdx.y;
    if (threadIdx.x == 0 && id < 8192) g_pf_span[kern][id][1] = gtime();
}
#define PF_TR(...) __VA_ARGS__
#else
#define PF_TR(...)
#endif

// ---- PTX helpers ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
// Bounded wait for the mbarrier phase with the given parity; false on timeout
// (0.25 s by %globaltimer, read every 256 polls, or 2^26 polls).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity) {
    const uint32_t a = smem_u32(b);
    unsigned long long t0 = 0;
    for (long long i = 0; i < WAIT_LIMIT; i++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.b32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255) == 255) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (i == 255) t0 = t;
            else if (t - t0 > WAIT_NS) return false;
        }
    }
    return false;
}
// Named barrier `id` over n threads returning the AND of their `v`.
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; barrier.red.and.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
// UMMA shared-memory descriptor, K-major, 128-byte swizzle: rows of 128 B,
// 8-row atoms 1024 B apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFF) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// bf16 x bf16 -> f32, both K-major, M = 128.
__device__ __forceinline__ uint32_t instr_desc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(PF_M >> 4) << 24);
}
// D (TMEM) (+)= A (TMEM, 128 lanes x 16 bf16 in 8 columns) . B^T (shared memory)
__device__ __forceinline__ void mma_bf16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
// This warp's 32 TMEM lanes, 16 / 4 consecutive 32-bit columns from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t v[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t v[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
        smem_u32(bar))
                 : "memory");
}
// Loads that leave the wait to the caller (tmem_ld_wait), so several are in
// flight at once.
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t r[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8_nw(uint32_t taddr, uint32_t r[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
}
// Waits for this thread's outstanding TMEM loads; the registers they wrote
// are passed through so no use of them is moved above the wait.
template <int N>
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[N]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < N; i++) asm volatile("" : "+r"(r[i]));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

// ---- copies -----------------------------------------------------------------
// TMA bulk copy global -> shared, completing on an mbarrier (this CTA only).
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    mbar_expect_tx(bar, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// One 2D box of the map at (x, y).
__device__ __forceinline__ void tma_tile2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ---- layout and conversion helpers ----------------------------------------------

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&p);
}
// Two quant bytes (k, k+1 of w, each < 128) as the bf16 pair (128 + q_k,
// 128 + q_k+1): 0x43 is the high byte of bf16 128, the quant is the mantissa.
template <int K>
__device__ __forceinline__ __nv_bfloat162 q_pair128(uint32_t w) {
    const uint32_t v = __byte_perm(w, 0x43434343u, K == 0 ? 0x4140u : 0x4342u);
    return *reinterpret_cast<const __nv_bfloat162 *>(&v);
}
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }

// ---- A operand, Q4_K ----------------------------------------------------------------
// Raw bytes of one matrix for one raw stage: Q4_K block b of 128 rows, one
// 2D TMA box of 128 rows x 144 bytes, [row][144] in shared memory (header at
// 0, quant chunk c of the block at 16 + 32c: elements 64c..64c+63).
// L2 policy for bytes read once per call (expert weights): evict them first,
// so the weight stream does not push the router, token rows and code out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// tma_tile2d with an L2 cache hint.
__device__ __forceinline__ void tma_tile2d_hint(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                                uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// bulk_copy with an L2 cache hint.
__device__ __forceinline__ void bulk_copy_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    mbar_expect_tx(bar, bytes);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void q4_issue(const CUtensorMap *map, int row0, uint32_t dst, int b, uint64_t *bar) {
    tma_tile2d_hint(dst, map, b * Q4K_BYTES, row0, bar, l2_evict_first());
}

// A dequantising thread owns one (row r, nibble half hh) of one matrix: in
// every stage it produces K elements 32hh..32hh+31 of row r (low nibbles for
// hh = 0, high for hh = 1) of chunk c, TMEM columns 16hh..16hh+15 of the
// A stage.
// Arithmetic is bf16 pairs: q exactly (bf16(128+q) - 128), then one fused
// q*bf16(d*sc) - bf16(dmin*m) rounded once to bf16. d*sc and dmin*m are the
// reference's fp32 products; rounding them to bf16 adds at most 2^-9 of
// |q*d*sc| + |dmin*m| to the bf16 operand's own rounding (2^-9 of |value|).
struct Q4Scales { uint32_t d2[4], nm2[4]; };  // bf16 pairs, sub-block 2c+hh for c = 0..3

// Decodes the row's block header (at the block's first stage) into the four
// scale pairs this thread uses in the block's four stages.
__device__ __forceinline__ void q4_scales(const uint8_t *raw, int r, int hh, Q4Scales &S) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * Q4K_BYTES);
    const uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    const float d = half_bits_ref(hdr.x & 0xFFFFu), dmin = half_bits_ref(hdr.x >> 16);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        int sc, mn;
        q4k_scale_min(s, 2 * c + hh, sc, mn);
        S.d2[c] = bf2_bits(__float2bfloat162_rn(__fmul_rn(d, (float)sc)));
        S.nm2[c] = bf2_bits(__float2bfloat162_rn(-__fmul_rn(dmin, (float)mn)));
    }
}

__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t v) { return *reinterpret_cast<const __nv_bfloat162 *>(&v); }

__device__ __forceinline__ void q4_deq(const uint8_t *raw, int c, int r, int hh, const Q4Scales &S,
                                       uint32_t out[16]) {
    const uint4 qa = *reinterpret_cast<const uint4 *>(raw + r * Q4K_BYTES + 16 + 32 * c);
    const uint4 qb = *reinterpret_cast<const uint4 *>(raw + r * Q4K_BYTES + 32 + 32 * c);
    // selects, not S.d2[c]: a runtime index would put S in local memory
    const __nv_bfloat162 d2 = as_bf2(c == 0 ? S.d2[0] : c == 1 ? S.d2[1] : c == 2 ? S.d2[2] : S.d2[3]);
    const __nv_bfloat162 nm2 = as_bf2(c == 0 ? S.nm2[0] : c == 1 ? S.nm2[1] : c == 2 ? S.nm2[2] : S.nm2[3]);
    const __nv_bfloat162 c128 = __float2bfloat162_rn(128.f);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int sh = 4 * hh;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t w = (qw[k] >> sh) & 0x0F0F0F0Fu;
        out[2 * k] = bf2_bits(__hfma2(__hsub2(q_pair128<0>(w), c128), d2, nm2));
        out[2 * k + 1] = bf2_bits(__hfma2(__hsub2(q_pair128<2>(w), c128), d2, nm2));
    }
}

// ---- A operand, Q6_K (from the raw slab in shared memory) ----------------------------
// 8 bytes at a 2-byte aligned shared-memory address.
__device__ __forceinline__ void lds_u64_2b(const uint8_t *p, uint32_t &lo, uint32_t &hi) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const unsigned sh = (unsigned)(a & 3) * 8;
    const uint32_t w0 = b[0], w1 = b[1], w2 = b[2];
    lo = __funnelshift_r(w0, w1, sh);
    hi = __funnelshift_r(w1, w2, sh);
}
// Half hb of a row's Q6_K blocks (block hb/2, elements 128 (hb%2) + 0..127:
// four quads of 32) for thread g: positions l = 8g..8g+7 of every quad, 32
// elements, each quant and scale byte read once. out[quad][j]: the bf16
// pair (l + 2j, l + 2j + 1) of the quad, (q-32) exactly times bf16(d*sc)
// rounded once (d*sc the reference's fp32 product).
__device__ __forceinline__ void q6_deq_half(const uint8_t *slab, int row_bytes, int hb, int r, int g,
                                            uint32_t out[4][4]) {
    const int half6 = hb & 1;
    const uint8_t *blk = slab + r * row_bytes + (hb >> 1) * Q6K_BYTES;
    uint32_t l0[2], l1[2], qh[2];
    lds_u64_2b(blk + half6 * 64 + 8 * g, l0[0], l0[1]);       // quads 0 (low nibbles) and 2 (high)
    lds_u64_2b(blk + half6 * 64 + 32 + 8 * g, l1[0], l1[1]);  // quads 1 and 3
    lds_u64_2b(blk + 128 + half6 * 32 + 8 * g, qh[0], qh[1]);  // two high bits of every quad
    const float d = half_bits_ref(*reinterpret_cast<const uint16_t *>(blk + 208));
    const uint8_t *sc = blk + 192 + half6 * 8 + (g >> 1);
    const __nv_bfloat162 c160 = __float2bfloat162_rn(160.f);
#pragma unroll
    for (int quad = 0; quad < 4; quad++) {
        const __nv_bfloat162 d2 = __float2bfloat162_rn(__fmul_rn(d, (float)(int8_t)sc[quad * 2]));
        const uint32_t *wl = (quad & 1) ? l1 : l0;
        const int nsh = quad >= 2 ? 4 : 0, hsh = 2 * quad;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint32_t q = ((wl[k] >> nsh) & 0x0F0F0F0Fu) | (((qh[k] >> hsh) & 0x03030303u) << 4);
            out[quad][2 * k] = bf2_bits(__hmul2(__hsub2(q_pair128<0>(q), c160), d2));
            out[quad][2 * k + 1] = bf2_bits(__hmul2(__hsub2(q_pair128<2>(q), c160), d2));
        }
    }
}

__device__ __forceinline__ int asg_token_p(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

// silu(g) * u = (g u / 2) (1 + tanh(g / 2)); the product is rounded to bf16
// next, and tanh.approx (relative error ~2^-11) is below that rounding. One
// MUFU and three FP32 operations, no branches: large |g| saturates tanh.
__device__ __forceinline__ float silu_mul(float g, float u) {
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
    const float h = 0.5f * g * u;
    return fmaf(h, t, h);
}

// Parity of the phase that completes the n-th use (n = 0, 1, ...) of a ring
// slot is n & 1; a producer refilling a slot for use n >= 1 waits for the
// consumer's release of use n-1, parity (n-1) & 1.

// ---- phase 1: gate/up (persistent) -----------------------------------------------------
// One CTA per SM loops over units (tile, 128 hidden rows), row block fastest,
// so CTAs running at the same time share a tile's x rows in L2. The raw
// Q4_K, x and A rings run on across unit boundaries, so the DRAM stream and
// the tensor core never drain between units.
//
// A thread waits about a hundred cycles on every tcgen05.mma it issues, so
// four threads issue them: issuer (m, p) the products of matrix m (gate,
// up) in the stages of parity p, into an accumulator of its own; the
// epilogue adds the two parities (a fixed order: deterministic). Units wider
// than 96 tokens have no room for four accumulators and use issuers (m, 0).
// TMEM (512 columns): two accumulator buffers of 192 columns. A unit of N <=
// 48 takes one buffer (accumulator (m, p) at 48 (2m + p)) and alternates with
// the next; N <= 96 takes both (at 96 (2m + p)); wider units take both
// without the parity split (gate at 0, up at 192). A stages at 384 + 64 s,
// matrix m at +32 m. 8 epilogue warps turn a finished unit's accumulators
// into h while the next unit accumulates.
constexpr int UP_EPI0 = 20;                  // first epilogue warp
constexpr int UP_NEPI = 8;                   // epilogue warps (2 per TMEM lane quarter)
constexpr int UP_ISS2 = UP_EPI0 + UP_NEPI;   // issuers (m, 1): warps 28, 29; (m, 0): warps 1, 3
constexpr int UP_THREADS = (UP_ISS2 + 2) * 32;
constexpr int UP_BUF = PF_NMAX;              // columns per accumulator buffer
constexpr int UP_NARROW = UP_BUF / 4;        // widest unit that fits one buffer (four accumulators)
constexpr int UP_SPLIT = UP_BUF / 2;         // widest unit with the parity split
constexpr int UP_A = 2 * UP_BUF;             // TMEM column of A stage 0 (64 columns each)
constexpr int UP_SMEM = 1024 + PF_STG * B_STAGE + PF_RAW * 2 * RAW4;

struct UpBars {
    uint64_t bfull[PF_STG], bempty[PF_STG];   // x: TMA -> MMA
    uint64_t rfull[PF_RAW], rempty[PF_RAW];   // raw Q4_K: TMA -> dequant
    uint64_t afull[PF_NA], aempty[PF_NA];     // A in TMEM: dequant -> MMA
    uint64_t cfull[2], cempty[2];             // accumulator buffers: MMA -> epilogue
};

// Accumulators of a unit: mask bit b set = buffer b used, split = parity
// split, col(m, p) = TMEM column of accumulator (m, p). `cur` is the buffer
// the next narrow unit takes. Every role walks the same unit sequence and so
// makes the same choices.
struct UpAcc {
    int mask, split, base, step;
    __device__ __forceinline__ uint32_t col(int m, int p) const { return base + (2 * m + p) * step; }
};
__device__ __forceinline__ UpAcc up_acc(int nn, int &cur) {
    UpAcc u;
    if (nn <= UP_NARROW) {
        u.mask = 1 << cur;
        u.split = 1;
        u.base = cur * UP_BUF;
        u.step = UP_NARROW;
        cur ^= 1;
        return u;
    }
    cur = 0;
    u.mask = 3;
    u.base = 0;
    u.split = nn <= UP_SPLIT;
    u.step = u.split ? UP_SPLIT : UP_BUF / 2;  // unsplit: (m, 0) at 192 m
    return u;
}

__global__ void __launch_bounds__(UP_THREADS, 1)
    prefill_up_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap umap,
                      const __grid_constant__ CUtensorMap gmap_sh, const __grid_constant__ CUtensorMap umap_sh) {
    extern __shared__ uint8_t psm_raw[];
    uint8_t *psm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ UpBars R;
    __shared__ uint32_t tslot;
    __shared__ __align__(16) __nv_bfloat16 epi_tile[UP_NEPI][16 * 40];  // per warp: 16 tokens x 32 rows (+pad)
    const int nblk = a.H / PF_M;
    const int n_units = *a.n_tiles * nblk;
    if ((int)blockIdx.x >= n_units) return;
    const int n_my = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    PF_TR(unsigned long long *tr = pf_tr(0); const unsigned long long tc0 = clock64(); unsigned long long tc;
          unsigned long long acc[20] = {};)
    const int nstages = a.D / PF_KS, nblocks = a.D / QK;
    uint8_t *bst = psm;                       // [PF_STG][B_STAGE]   1024-aligned
    uint8_t *raw = bst + PF_STG * B_STAGE;    // [PF_RAW][gate raw | up raw]
    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STG; i++) {
            mbar_init(&R.bfull[i], 1);
            mbar_init(&R.bempty[i], 2);
        }
        for (int i = 0; i < PF_RAW; i++) {
            mbar_init(&R.rfull[i], 1);
            mbar_init(&R.rempty[i], PF_NDQW);
        }
        for (int i = 0; i < PF_NA; i++) {
            mbar_init(&R.afull[i], PF_NDQW);
            mbar_init(&R.aempty[i], 2);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&R.cfull[i], 4);
            mbar_init(&R.cempty[i], UP_NEPI);
        }
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 512);  // syncs the CTA
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = true;
    if (warp == 0) {
        // x producer: per stage the unit's nn rows of xg, in 16-row boxes
        if (lane == 0) {
            int g = 0;
            for (int k = 0; k < n_my && ok; k++) {
                const int tile = ((int)blockIdx.x + k * (int)gridDim.x) / nblk;
                const int s0 = a.tile_start[tile], nn = (a.tile_n[tile] + 15) & ~15;
                for (int i = 0; i < nstages && ok; i++, g++) {
                    const int sb = g % PF_STG, use = g / PF_STG;
                    PF_TR(tc = clock64();)
                    if (use > 0) ok = mbar_wait(&R.bempty[sb], (use - 1) & 1);
                    PF_TR(acc[4] += clock64() - tc;)
                    if (!ok) break;
                    mbar_expect_tx(&R.bfull[sb], nn * 128);
                    const uint32_t dst = smem_u32(bst + sb * B_STAGE);
                    for (int q = 0; q < nn / B_ROWS; q++)
                        tma_tile2d(dst + q * B_ROWS * 128, &xmap, i * PF_KS, s0 + q * B_ROWS, &R.bfull[sb]);
                }
            }
        }
    } else if (warp == 2) {
        // raw Q4_K producer: gate and up block i of the unit's 128 rows, up
        // to PF_RAW blocks ahead
        if (lane == 0) {
            int g = 0;
            for (int k = 0; k < n_my && ok; k++) {
                const int u = (int)blockIdx.x + k * (int)gridDim.x, tile = u / nblk, m0 = (u - tile * nblk) * PF_M;
                const int e = a.slot_expert[a.tile_slot[tile]];
                const CUtensorMap *gm = e == a.E ? &gmap_sh : &gmap, *um = e == a.E ? &umap_sh : &umap;
                const int row0 = (e == a.E ? 0 : e * a.H) + m0;
                for (int i = 0; i < nblocks && ok; i++, g++) {
                    const int sr = g % PF_RAW, use = g / PF_RAW;
                    PF_TR(tc = clock64();)
                    if (use > 0) ok = mbar_wait(&R.rempty[sr], (use - 1) & 1);
                    PF_TR(acc[5] += clock64() - tc;)
                    if (!ok) break;
                    mbar_expect_tx(&R.rfull[sr], 2 * RAW4);
                    const uint32_t rd = smem_u32(raw + sr * 2 * RAW4);
                    q4_issue(gm, row0, rd, i, &R.rfull[sr]);
                    q4_issue(um, row0, rd + RAW4, i, &R.rfull[sr]);
                }
            }
        }
    } else if (warp == 1 || warp == 3 || warp >= UP_ISS2) {
        // MMA issuer (m, p); every issuer waits for the buffers' release
        // before committing to their cfull, so no arrival lands in an
        // earlier phase
        const int mat = warp == 3 || warp == UP_ISS2 + 1, par = warp >= UP_ISS2;
        if (lane == 0) {
            int g = 0, cur = 0, uses[2] = {0, 0};
            for (int k = 0; k < n_my && ok; k++) {
                const int tile = ((int)blockIdx.x + k * (int)gridDim.x) / nblk;
                const int nn = (a.tile_n[tile] + 15) & ~15;
                const uint32_t idesc = instr_desc(nn);
                const UpAcc ua = up_acc(nn, cur);
                PF_TR(tc = clock64();)
                for (int b = 0; b < 2 && ok; b++)
                    if ((ua.mask >> b) & 1) {
                        if (uses[b] > 0) ok = mbar_wait(&R.cempty[b], (uses[b] - 1) & 1);
                    }
                PF_TR(acc[14] += clock64() - tc;)
                if (!ok) break;
                tc_fence_after();
                const uint32_t dacc = tbase + ua.col(mat, par);
                const bool active = ua.split || par == 0;
                for (int i = 0; i < nstages && ok; i++, g++) {
                    if (!active || (ua.split && (i & 1) != par)) continue;
                    const int sa = g % PF_NA, sb = g % PF_STG;
                    PF_TR(tc = clock64();)
                    ok = mbar_wait(&R.afull[sa], (g / PF_NA) & 1);
                    PF_TR(acc[6] += clock64() - tc; tc = clock64();)
                    ok = ok && mbar_wait(&R.bfull[sb], (g / PF_STG) & 1);
                    PF_TR(acc[7] += clock64() - tc; tc = clock64();)
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t bb = smem_u32(bst + sb * B_STAGE), ta = tbase + UP_A + sa * 64 + mat * 32;
                    const int first = ua.split ? 2 : 1;  // stages before this accumulator's second
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; kk++)
                        mma_bf16_ta(dacc, ta + kk * 8, sw128_desc(bb + kk * 32), idesc, i >= first || kk != 0);
                    mma_commit(&R.aempty[sa]);
                    mma_commit(&R.bempty[sb]);
                    PF_TR(acc[16] += clock64() - tc;)
                }
                for (int b = 0; b < 2; b++)
                    if ((ua.mask >> b) & 1) {
                        mma_commit(&R.cfull[b]);  // arrives once this issuer's MMAs complete
                        uses[b]++;
                    }
            }
        }
    } else if (warp >= PF_DQ0 / 32 && warp < UP_EPI0) {
        // dequantisers: warp w owns TMEM lanes (= weight rows) 32*(w%4)..,
        // matrix and nibble half from (w-4)/4
        const int grp = (warp - PF_DQ0 / 32) >> 2, mat = grp >> 1, hh = grp & 1;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t t_st = tbase + ((uint32_t)((warp & 3) * 32) << 16) + UP_A + mat * 32 + hh * 16;
        Q4Scales S;
        int g = 0, gr = 0;  // A stages, raw blocks
        for (int k = 0; k < n_my && ok; k++) {
            for (int i = 0; i < nblocks && ok; i++, gr++) {
                const int sr = gr % PF_RAW;
                PF_TR(tc = clock64();)
                ok = mbar_wait(&R.rfull[sr], (gr / PF_RAW) & 1);
                PF_TR(if (threadIdx.x == PF_DQ0) acc[8] += clock64() - tc;)
                if (!ok) break;
                const uint8_t *rw = raw + sr * 2 * RAW4 + mat * RAW4;
                q4_scales(rw, r, hh, S);
                for (int c = 0; c < QK / PF_KS && ok; c++, g++) {
                    const int sa = g % PF_NA;
                    PF_TR(tc = clock64();)
                    if (g >= PF_NA) ok = mbar_wait(&R.aempty[sa], (g / PF_NA - 1) & 1);
                    PF_TR(if (threadIdx.x == PF_DQ0) acc[9] += clock64() - tc; tc = clock64();)
                    if (!ok) break;
                    tc_fence_after();
                    uint32_t v[16];
                    q4_deq(rw, c, r, hh, S, v);
                    tmem_st16(t_st + sa * 64, v);
                    tmem_st_wait();
                    PF_TR(if (threadIdx.x == PF_DQ0) acc[10] += clock64() - tc;)
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&R.afull[sa]);
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&R.rempty[sr]);
            }
        }
    } else if (warp >= UP_EPI0) {
        // epilogue: h = bf16(silu(gate) * up) for the unit's 128 rows. Warp
        // (q, half) reads TMEM lanes 32q.. and alternate 16-token chunks,
        // turns each 32-row x 16-token block around in shared memory and
        // stores 16-byte pieces of the tokens' h rows.
        const int q = warp & 3, half = (warp - UP_EPI0) >> 2, ew = warp - UP_EPI0;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        __nv_bfloat16 *blk = epi_tile[ew];  // [16 tokens][40]
        int cur = 0, uses[2] = {0, 0};
        for (int k = 0; k < n_my && ok; k++) {
            const int u = (int)blockIdx.x + k * (int)gridDim.x, tile = u / nblk, m0 = (u - tile * nblk) * PF_M;
            const int s0 = a.tile_start[tile], n = a.tile_n[tile], nn = (n + 15) & ~15;
            const UpAcc ua = up_acc(nn, cur);
            const int mask = ua.mask;
            bool got = true;
            for (int b = 0; b < 2; b++)
                if ((mask >> b) & 1) got = got && mbar_wait(&R.cfull[b], uses[b] & 1);
            // every epilogue warp reaches this barrier (its waits are
            // bounded), so they leave together on a timeout
            PF_TR(tc = clock64();)
            ok = bar_and(2, UP_NEPI * 32, got);
            PF_TR(if (threadIdx.x == UP_EPI0 * 32) acc[17] += clock64() - tc; tc = clock64();)
            if (!ok) break;
            tc_fence_after();
            const uint32_t tg = tbase + lane_off + ua.col(0, 0), tu = tbase + lane_off + ua.col(1, 0);
            const uint32_t tg1 = tbase + lane_off + ua.col(0, 1), tu1 = tbase + lane_off + ua.col(1, 1);
            __nv_bfloat16 *hrow = a.hb + (size_t)s0 * a.H + m0 + q * 32 + 8 * (lane & 3);
            for (int j0 = half * 16; j0 < n; j0 += 32) {
                if (ua.split) {
#pragma unroll
                    for (int jh = 0; jh < 16; jh += 8) {
                        uint32_t r[32];
                        tmem_ld8_nw(tg + j0 + jh, r);
                        tmem_ld8_nw(tu + j0 + jh, r + 8);
                        tmem_ld8_nw(tg1 + j0 + jh, r + 16);
                        tmem_ld8_nw(tu1 + j0 + jh, r + 24);
                        tmem_ld_wait(r);
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float gv = __uint_as_float(r[j]) + __uint_as_float(r[16 + j]);
                            const float uv = __uint_as_float(r[8 + j]) + __uint_as_float(r[24 + j]);
                            blk[(jh + j) * 40 + lane] = __float2bfloat16_rn(silu_mul(gv, uv));
                        }
                    }
                } else {
                    uint32_t r[32];
                    tmem_ld16_nw(tg + j0, r);
                    tmem_ld16_nw(tu + j0, r + 16);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        blk[j * 40 + lane] =
                            __float2bfloat16_rn(silu_mul(__uint_as_float(r[j]), __uint_as_float(r[16 + j])));
                }
                __syncwarp();
                // lane: token j0 + (lane >> 2) + 8 it, rows 8*(lane & 3)..+7
#pragma unroll
                for (int it = 0; it < 2; it++) {
                    const int jj = (lane >> 2) + 8 * it;
                    if (j0 + jj < n)
                        *reinterpret_cast<uint4 *>(hrow + (size_t)(j0 + jj) * a.H) =
                            *reinterpret_cast<const uint4 *>(blk + jj * 40 + 8 * (lane & 3));
                }
                __syncwarp();
            }
            PF_TR(if (threadIdx.x == UP_EPI0 * 32) acc[18] += clock64() - tc;)
            tc_fence_before();
            __syncwarp();
            for (int b = 0; b < 2; b++)
                if ((mask >> b) & 1) {
                    if (lane == 0) mbar_arrive(&R.cempty[b]);
                    uses[b]++;
                }
        }
    }
    PF_TR(if (tr) {
        _Pragma("unroll") for (int i = 4; i < 20; i++) if (acc[i]) atomicAdd(&tr[i], acc[i]);
    })
    ok = __syncthreads_and(ok);
    if (!ok && threadIdx.x == 0) atomicExch(a.err, 1);
    PF_TR(if (tr && threadIdx.x == 0) { tr[2] = clock64() - tc0; tr[13] = n_my; })
    tmem_free(tbase, 512);
    PF_TR(if (tr && threadIdx.x == 0) tr[3] = clock64() - tc0; pf_end(0);)
}

// ---- phase 2: down + weighted combine (persistent) -----------------------------
// One CTA per SM loops over units (tile, 128 output rows), output-row block
// fastest, so the CTAs running at the same time share a tile's h rows in L2.
// The unit's 128 Q6_K rows (one contiguous, 16-byte aligned slab, 128 x 420 B
// at H = 512) come in one bulk copy into one of two slab buffers while the
// previous unit computes; the tensor core accumulates into one of two TMEM
// accumulators while 8 epilogue warps add the other one's w * y into out.
// Dequantising thread (r, g) decodes positions 8g..8g+7 of all four quads of
// a half block (two A stages at once, every byte read once). Two threads
// issue the MMAs (a thread waits about a hundred cycles per tcgen05.mma): for
// units of N <= 96, issuer p takes the stages of parity p into an accumulator
// of its own (columns +0 and +96 of the unit's buffer) and the epilogue adds
// the two; wider units use issuer 0 alone.
// TMEM: accumulators [0,192) and [192,384), four A stages [384,512).
constexpr int DN_EPI0 = 20;                 // first epilogue warp (warps 1 and 3 issue MMAs)
constexpr int DN_NEPI = 8;                  // epilogue warps (2 per TMEM lane quarter)
constexpr int DN_THREADS = (DN_EPI0 + DN_NEPI) * 32;
constexpr int DN_ACC1 = PF_NMAX;            // TMEM column of the second accumulator
constexpr int DN_SPLIT = PF_NMAX / 2;       // widest unit with the parity split
constexpr int DN_A = 2 * PF_NMAX;           // TMEM column of A stage 0 (32 columns each)
constexpr int DN_NA = 4;                    // A stages (two half blocks in flight)

__host__ __device__ inline int down_slab_bytes(int H) { return PF_M * (H / QK) * Q6K_BYTES; }
__host__ __device__ inline int down_smem(int H) { return 1024 + PF_STG * B_STAGE + 2 * down_slab_bytes(H); }

struct DownBars {
    uint64_t bfull[PF_STG], bempty[PF_STG];  // B: TMA -> MMA
    uint64_t afull[DN_NA], aempty[DN_NA];    // A in TMEM: dequant -> MMA
    uint64_t sfull[2], sempty[2];            // Q6_K slabs: bulk copy -> dequant
    uint64_t cfull[2], cempty[2];            // accumulators: MMA -> epilogue
};

__global__ void __launch_bounds__(DN_THREADS, 1)
    prefill_down_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap hmap) {
    extern __shared__ uint8_t psm_raw[];
    uint8_t *psm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ DownBars R;
    __shared__ uint32_t tslot;
    __shared__ float epi_tile[DN_NEPI * 16 * 33];     // per epilogue warp: 16 tokens x 32 rows
    __shared__ int epi_tok[PF_NMAX];                  // the unit's tokens
    __shared__ float epi_w[PF_NMAX];                  // and their weights
    const int nblk = a.D / PF_M;
    const int n_units = *a.n_tiles * nblk;
    if ((int)blockIdx.x >= n_units) return;
    const int n_my = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    PF_TR(unsigned long long *tr = pf_tr(1); const unsigned long long tc0 = clock64(); unsigned long long tc;
          unsigned long long acc[20] = {};)
    const int TK = a.T * a.K;
    const int row_bytes = (a.H / QK) * Q6K_BYTES, slab_bytes = PF_M * row_bytes;
    const size_t exp_bytes = (size_t)row_bytes * a.D;
    const int nstages = a.H / PF_KS;
    uint8_t *bst = psm;                        // [PF_STG][B_STAGE]
    uint8_t *slab = bst + PF_STG * B_STAGE;    // [2][slab_bytes], 16-byte aligned
    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STG; i++) {
            mbar_init(&R.bfull[i], 1);
            mbar_init(&R.bempty[i], 1);
        }
        for (int i = 0; i < DN_NA; i++) {
            mbar_init(&R.afull[i], PF_NDQW);
            mbar_init(&R.aempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&R.sfull[i], 1);
            mbar_init(&R.sempty[i], PF_NDQW);
            mbar_init(&R.cfull[i], 2);
            mbar_init(&R.cempty[i], DN_NEPI);
        }
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 512);  // syncs the CTA
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = true;
    if (warp == 2) {
        // slab producer: the unit's 128 Q6_K rows in one bulk copy, as soon
        // as a slab buffer is free
        if (lane == 0) {
            for (int k = 0; k < n_my && ok; k++) {
                const int u = (int)blockIdx.x + k * (int)gridDim.x, tile = u / nblk, n0 = (u - tile * nblk) * PF_M;
                const int e = a.slot_expert[a.tile_slot[tile]];
                const int sb = k & 1;
                if (k >= 2) ok = mbar_wait(&R.sempty[sb], ((k >> 1) - 1) & 1);
                if (!ok) break;
                bulk_copy_hint(slab + sb * slab_bytes, (e == a.E ? a.down_sh : a.down + e * exp_bytes) + (size_t)n0 * row_bytes,
                               slab_bytes, &R.sfull[sb], l2_evict_first());
            }
        }
    } else if (warp == 0) {
        // h producer: the unit's h rows per stage
        if (lane == 0) {
            int g = 0;  // stage counter across units
            for (int k = 0; k < n_my && ok; k++) {
                const int tile = ((int)blockIdx.x + k * (int)gridDim.x) / nblk;
                const int s0 = a.tile_start[tile];
                const int nn = (a.tile_n[tile] + 15) & ~15;
                for (int i = 0; i < nstages && ok; i++, g++) {
                    const int rb = g % PF_STG, use = g / PF_STG;
                    if (use > 0) ok = mbar_wait(&R.bempty[rb], (use - 1) & 1);
                    if (!ok) break;
                    mbar_expect_tx(&R.bfull[rb], nn * 128);
                    const uint32_t dst = smem_u32(bst + rb * B_STAGE);
                    for (int q = 0; q < nn / B_ROWS; q++)
                        tma_tile2d(dst + q * B_ROWS * 128, &hmap, i * PF_KS, s0 + q * B_ROWS, &R.bfull[rb]);
                }
            }
        }
    } else if (warp == 1 || warp == 3) {
        // MMA issuer p: unit k accumulates into TMEM buffer k % 2; both
        // issuers wait for the buffer's release and commit to its cfull
        const int par = warp == 3;
        if (lane == 0) {
            int g = 0;
            for (int k = 0; k < n_my && ok; k++) {
                const int tile = ((int)blockIdx.x + k * (int)gridDim.x) / nblk;
                const int nn = (a.tile_n[tile] + 15) & ~15;
                const uint32_t idesc = instr_desc(nn);
                const bool split = nn <= DN_SPLIT;
                const int ab = k & 1;
                PF_TR(tc = clock64();)
                if (k >= 2) ok = mbar_wait(&R.cempty[ab], ((k >> 1) - 1) & 1);
                PF_TR(acc[14] += clock64() - tc;)
                if (!ok) break;
                tc_fence_after();
                const uint32_t dacc = tbase + ab * DN_ACC1 + par * DN_SPLIT;
                const int first = split ? 2 : 1;  // stages before this accumulator's second
                for (int i = 0; i < nstages && ok; i++, g++) {
                    if (split ? (i & 1) != par : par != 0) continue;
                    const int sa = g % DN_NA, sb = g % PF_STG;
                    PF_TR(tc = clock64();)
                    ok = mbar_wait(&R.afull[sa], (g / DN_NA) & 1);
                    PF_TR(acc[6] += clock64() - tc; tc = clock64();)
                    ok = ok && mbar_wait(&R.bfull[sb], (g / PF_STG) & 1);
                    PF_TR(acc[7] += clock64() - tc; tc = clock64();)
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t bb = smem_u32(bst + sb * B_STAGE), ta = tbase + DN_A + sa * 32;
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; kk++)
                        mma_bf16_ta(dacc, ta + kk * 8, sw128_desc(bb + kk * 32), idesc, i >= first || kk != 0);
                    mma_commit(&R.aempty[sa]);
                    mma_commit(&R.bempty[sb]);
                    PF_TR(acc[16] += clock64() - tc;)
                }
                mma_commit(&R.cfull[ab]);  // arrives once this issuer's MMAs complete
                // an issuer that sat out a unit waits for it to finish: the
                // next unit's buffer wait covers the unit before, not this
                // one, and running on could put its A waits two phases ahead
                if (!split && par != 0) ok = mbar_wait(&R.cfull[ab], (k >> 1) & 1);
            }
        }
    } else if (warp >= PF_DQ0 / 32 && warp < DN_EPI0) {
        // dequantisers: warp w owns TMEM lanes (= rows) 32*(w%4).. of A and
        // positions 8g..8g+7 (g = (w-4)/4) of every quad: per half block h
        // it fills A stages 2h (quads 0, 1) and 2h + 1 (quads 2, 3), columns
        // 4g.. and 16 + 4g.. of each
        const int gq = (warp - PF_DQ0 / 32) >> 2;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t t_st = tbase + ((uint32_t)((warp & 3) * 32) << 16) + DN_A + 4 * gq;
        const int nhalf = nstages / 2;
        int g = 0;  // A stages
        for (int k = 0; k < n_my && ok; k++) {
            const int sb = k & 1;
            PF_TR(tc = clock64();)
            ok = mbar_wait(&R.sfull[sb], (k >> 1) & 1);
            PF_TR(if (threadIdx.x == PF_DQ0) acc[8] += clock64() - tc;)
            const uint8_t *sl = slab + sb * slab_bytes;
            for (int h = 0; h < nhalf && ok; h++, g += 2) {
                const int s0 = g % DN_NA;  // stages s0, s0 + 1 (DN_NA is even)
                PF_TR(tc = clock64();)
                if (g >= DN_NA)
                    ok = mbar_wait(&R.aempty[s0], (g / DN_NA - 1) & 1) &&
                         mbar_wait(&R.aempty[s0 + 1], (g / DN_NA - 1) & 1);
                PF_TR(if (threadIdx.x == PF_DQ0) acc[9] += clock64() - tc; tc = clock64();)
                if (!ok) break;
                tc_fence_after();
                uint32_t v[4][4];
                q6_deq_half(sl, row_bytes, h, r, gq, v);
#pragma unroll
                for (int quad = 0; quad < 4; quad++)
                    tmem_st4(t_st + (s0 + (quad >> 1)) * 32 + (quad & 1) * 16, v[quad]);
                tmem_st_wait();
                PF_TR(if (threadIdx.x == PF_DQ0) acc[10] += clock64() - tc;)
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&R.afull[s0]);
                    mbar_arrive(&R.afull[s0 + 1]);
                }
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&R.sempty[sb]);  // done reading this slab
        }
    } else if (warp >= DN_EPI0) {
        // epilogue: out[token] += w * y for the 128 rows of the unit. Warp
        // (q, half) reads TMEM lanes 32q.. and alternate 16-token chunks,
        // turns each 32-row x 16-token block around in shared memory and
        // adds whole 16-byte row pieces (red.global.add.v4.f32).
        const int q = warp & 3, half = (warp - DN_EPI0) >> 2, ew = warp - DN_EPI0;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        float *blk = epi_tile + ew * 16 * 33;  // [16 tokens][32 rows + 1]
        for (int k = 0; k < n_my && ok; k++) {
            const int u = (int)blockIdx.x + k * (int)gridDim.x, tile = u / nblk, n0 = (u - tile * nblk) * PF_M;
            const int s0 = a.tile_start[tile], n = a.tile_n[tile], nn = (n + 15) & ~15;
            const int ab = k & 1;
            // every epilogue warp reaches this barrier (its wait is bounded),
            // so they leave together on a timeout; it also marks the
            // previous unit's readers done
            PF_TR(tc = clock64();)
            ok = bar_and(2, DN_NEPI * 32, mbar_wait(&R.cfull[ab], (k >> 1) & 1));
            PF_TR(if (threadIdx.x == DN_EPI0 * 32) acc[17] += clock64() - tc; tc = clock64();)
            if (!ok) break;
            tc_fence_after();
            // token and weight of each tile row, shared by the epilogue warps
            for (int j = ew * 32 + lane; j < n; j += DN_NEPI * 32) {
                const int asg = __ldg(a.assign + s0 + j);
                const int t = asg_token_p(asg, TK, a.K);
                epi_tok[j] = t;
                epi_w[j] = asg < TK ? __ldg(a.w + asg) : (a.shared_gate ? __ldg(a.gsc + t) : 1.0f);
            }
            asm volatile("bar.sync 2, %0;" ::"n"(DN_NEPI * 32) : "memory");
            const uint32_t tacc = tbase + lane_off + ab * DN_ACC1;
            const bool split = nn <= DN_SPLIT;
            float *orow = a.out + n0 + q * 32 + 4 * (lane & 7);
            for (int j0 = half * 16; j0 < n; j0 += 32) {
                float y[16];
                {
                    uint32_t r[32];
                    tmem_ld16_nw(tacc + j0, r);
                    if (split) tmem_ld16_nw(tacc + DN_SPLIT + j0, r + 16);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        y[j] = split ? __uint_as_float(r[j]) + __uint_as_float(r[16 + j]) : __uint_as_float(r[j]);
                }
#pragma unroll
                for (int j = 0; j < 16; j++) blk[j * 33 + lane] = y[j];
                __syncwarp();
                // lane: token j0 + (lane >> 3) + 4 it, rows 4*(lane & 7)..+3
#pragma unroll
                for (int it = 0; it < 4; it++) {
                    const int jj = (lane >> 3) + 4 * it;
                    if (j0 + jj < n) {
                        const float wv = epi_w[j0 + jj];
                        const float *src = blk + jj * 33 + 4 * (lane & 7);
                        float *dst = orow + (size_t)epi_tok[j0 + jj] * a.D;
                        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(wv * src[0]),
                                     "f"(wv * src[1]), "f"(wv * src[2]), "f"(wv * src[3])
                                     : "memory");
                    }
                }
                __syncwarp();
            }
            PF_TR(if (threadIdx.x == DN_EPI0 * 32) acc[18] += clock64() - tc;)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&R.cempty[ab]);
        }
    }
    PF_TR(if (tr) {
        _Pragma("unroll") for (int i = 4; i < 20; i++) if (acc[i]) atomicAdd(&tr[i], acc[i]);
    })
    ok = __syncthreads_and(ok);
    if (!ok && threadIdx.x == 0) atomicExch(a.err, 1);
    PF_TR(if (tr && threadIdx.x == 0) { tr[2] = clock64() - tc0; tr[13] = n_my; })
    tmem_free(tbase, 512);
    PF_TR(if (tr && threadIdx.x == 0) tr[3] = clock64() - tc0; pf_end(1);)
}

// ---- helpers: x to bf16, tile list ---------------------------------------------
// x rows of every assignment, as bf16, in slot order: xg[p] = bf16(x[token of
// assign[p]]). One warp per row.
__global__ void gather_rows_kernel(const float *__restrict__ x, const int *__restrict__ assign,
                                   const int *n_slots, const int *slot_start, int TK, int K, int D,
                                   __nv_bfloat16 *__restrict__ xg) {
    const int rows = slot_start[*n_slots];
    const int lane = threadIdx.x & 31;
    for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < rows; p += (gridDim.x * blockDim.x) >> 5) {
        // 8 elements per lane and step: two 16-byte loads, one 16-byte store
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)asg_token_p(assign[p], TK, K) * D);
        uint4 *dst = reinterpret_cast<uint4 *>(xg + (size_t)p * D);
        for (int c = lane; c < D / 8; c += 32) {
            const float4 v = __ldg(src + 2 * c), u = __ldg(src + 2 * c + 1);
            dst[c] = make_uint4(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w), pack_bf16(u.x, u.y), pack_bf16(u.z, u.w));
        }
    }
}

// The same for token rows that are already bf16 (rows received from peers).
__global__ void gather_rows_bf16_kernel(const __nv_bfloat16 *__restrict__ x, const int *__restrict__ assign,
                                        const int *n_slots, const int *slot_start, int TK, int K, int D,
                                        __nv_bfloat16 *__restrict__ xg) {
    const int rows = slot_start[*n_slots];
    const int lane = threadIdx.x & 31;
    for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < rows; p += (gridDim.x * blockDim.x) >> 5) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)asg_token_p(assign[p], TK, K) * D);
        uint4 *dst = reinterpret_cast<uint4 *>(xg + (size_t)p * D);
        for (int c = lane; c < D / 8; c += 32) dst[c] = __ldcg(src + c);
    }
}

// One block: split every slot into tiles of at most 256 tokens.
__global__ void __launch_bounds__(1024) tile_plan_kernel(const int *n_slots, const int *slot_start, int *n_tiles,
                                                         int *tile_slot, int *tile_start, int *tile_n) {
    // thread u owns slot u (at most 1025 slots: E <= 1024 routed experts +
    // the shared one, so 1024 threads and one extra pass for the last)
    __shared__ int wsum[32], total;
    const int ns = *n_slots, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    int carry = 0;
    for (int u0 = 0; u0 < ns; u0 += blockDim.x) {
        const int u = u0 + tid;
        const int nt = u < ns ? (slot_start[u + 1] - slot_start[u] + PF_NMAX - 1) / PF_NMAX : 0;
        int inc = nt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        if (lane == 31) wsum[wid] = inc;
        __syncthreads();
        if (wid == 0) {
            const int nw = blockDim.x >> 5;
            const int w = lane < nw ? wsum[lane] : 0;
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += v;
            }
            if (lane < nw) wsum[lane] = wi - w;
            if (lane == 31) total = wi;
        }
        __syncthreads();
        const int base = carry + wsum[wid] + inc - nt;
        if (u < ns) {
            const int st = slot_start[u];
            for (int k = 0; k < nt; k++) {
                tile_slot[base + k] = u;
                tile_start[base + k] = st + k * PF_NMAX;
                tile_n[base + k] = min(PF_NMAX, slot_start[u + 1] - st - k * PF_NMAX);
            }
        }
        carry += total;
        __syncthreads();  // wsum and total are rewritten next pass
    }
    if (tid == 0) *n_tiles = carry;
}

int prefill_max_tiles(int T, int K, int E) {
    const int assignments = T * K + T;
    const int slots = (T * K < E ? T * K : E) + 1;
    return assignments / PF_NMAX + slots + 1;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Row-major [rows][cols] bf16 tensor, boxes of 64 columns x box_rows rows,
// 128-byte swizzle.
static int encode_bf16_2d(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return OFB_ECUDA;
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)PF_KS, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (bf16) failed (%d)", (int)r);
        return OFB_ECUDA;
    }
    return OFB_OK;
}

// Q4_K rows as a 2D byte tensor [rows][row bytes]; boxes of one 144-byte
// block x 128 rows (x = block * 144, a multiple of 16 bytes).
static int encode_q4_rows(CUtensorMap *map, const void *base, int D, uint64_t rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return OFB_ECUDA;
    }
    if (reinterpret_cast<uintptr_t>(base) & 15) {
        set_error("Q4_K expert tensors must be 16-byte aligned for the prefill kernels");
        return OFB_EINVAL;
    }
    const uint64_t row_bytes = (uint64_t)(D / QK) * Q4K_BYTES;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {Q4K_BYTES, (cuuint32_t)PF_M};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (Q4_K rows) failed (%d)", (int)r);
        return OFB_ECUDA;
    }
    return OFB_OK;
}

int launch_prefill(const LayerArgs &la, const float *x, int *n_slots, __nv_bfloat16 *xb, __nv_bfloat16 *hb,
                   int *tiles, bool tiles_ready, int *err, cudaStream_t s, cudaEvent_t before, cudaEvent_t between) {
    const int T = la.T, D = la.D, H = la.H;
    const int max_tiles = prefill_max_tiles(T, la.K, la.E);
    const int n_asg = T * la.K + T;
    int *n_tiles = tiles, *tile_slot = tiles + 1, *tile_start = tile_slot + max_tiles,
        *tile_n = tile_start + max_tiles;
    CUtensorMap xmap, hmap, gmap, umap, gmap_sh, umap_sh;
    int st;
    if ((st = encode_bf16_2d(&xmap, xb, D, n_asg, B_ROWS))) return st;  // 64 x 16 boxes
    if ((st = encode_bf16_2d(&hmap, hb, H, n_asg, B_ROWS))) return st;
    if ((st = encode_q4_rows(&gmap, la.gate, D, (uint64_t)la.E * H))) return st;
    if ((st = encode_q4_rows(&umap, la.up, D, (uint64_t)la.E * H))) return st;
    if (la.has_shared) {
        if ((st = encode_q4_rows(&gmap_sh, la.gate_sh, D, H))) return st;
        if ((st = encode_q4_rows(&umap_sh, la.up_sh, D, H))) return st;
    } else {
        gmap_sh = gmap;  // never read: no slot names the shared expert
        umap_sh = umap;
    }
    if (la.xb_in)
        gather_rows_bf16_kernel<<<148 * 8, 256, 0, s>>>(la.xb_in, la.assign, n_slots, la.slot_start, T * la.K, la.K,
                                                         D, xb);
    else
        gather_rows_kernel<<<148 * 8, 256, 0, s>>>(x, la.assign, n_slots, la.slot_start, T * la.K, la.K, D, xb);
    if (!tiles_ready) tile_plan_kernel<<<1, 1024, 0, s>>>(n_slots, la.slot_start, n_tiles, tile_slot, tile_start, tile_n);
    PrefillArgs a;
    a.T = T; a.D = D; a.H = H; a.E = la.E; a.K = la.K;
    a.shared_gate = la.shared_gate;
    a.gate = la.gate; a.up = la.up; a.down = la.down;
    a.gate_sh = la.gate_sh; a.up_sh = la.up_sh; a.down_sh = la.down_sh;
    a.slot_expert = la.slot_expert; a.slot_start = la.slot_start; a.assign = la.assign;
    a.n_tiles = n_tiles; a.tile_slot = tile_slot; a.tile_start = tile_start; a.tile_n = tile_n;
    a.hb = hb; a.w = la.w; a.gsc = la.gsc; a.out = la.out; a.err = err;
    const int smem_up = UP_SMEM;
    const int smem_dn = down_smem(H);
    static size_t attr_up[64], attr_dn[64];
    cudaError_t ea = ensure_dyn_smem(prefill_up_kernel, (size_t)smem_up, attr_up);
    if (ea == cudaSuccess) ea = ensure_dyn_smem(prefill_down_kernel, (size_t)smem_dn, attr_dn);
    if (ea != cudaSuccess) return cuda_status(ea, "prefill smem attribute");
    // out starts as the residual (or zero); the down kernel adds w * y into it
    cudaError_t e;
    if (!la.resid) e = cudaMemsetAsync(la.out, 0, (size_t)T * D * sizeof(float), s);
    else if (la.resid != la.out)
        e = cudaMemcpyAsync(la.out, la.resid, (size_t)T * D * sizeof(float), cudaMemcpyDeviceToDevice, s);
    else e = cudaSuccess;
    if (e != cudaSuccess) return cuda_status(e, "prefill out init");
    if (before) cudaEventRecord(before, s);
    const int sms = sm_count();
    const int up_units = max_tiles * (H / PF_M);
    prefill_up_kernel<<<up_units < sms ? up_units : sms, UP_THREADS, smem_up, s>>>(a, xmap, gmap, umap, gmap_sh,
                                                                                     umap_sh);
    if (between) cudaEventRecord(between, s);
    const int dn_units = max_tiles * (D / PF_M);
    prefill_down_kernel<<<dn_units < sms ? dn_units : sms, DN_THREADS, smem_dn, s>>>(a, hmap);
    OFB_CHECK_LAUNCH("prefill kernels");
    return OFB_OK;
}

}  // namespace ofb

#ifdef OFB_PF_TRACE
extern "C" int ofb_debug_prefill_trace(unsigned long long *host, unsigned long long *span) {
    if (cudaMemcpyFromSymbol(host, ofb::g_pf_trace, sizeof(ofb::g_pf_trace)) != cudaSuccess) return 1;
    return cudaMemcpyFromSymbol(span, ofb::g_pf_span, sizeof(ofb::g_pf_span)) == cudaSuccess ? 0 : 1;
}
#endif
