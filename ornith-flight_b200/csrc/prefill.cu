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
//  * B (token rows): TMA. The up GEMM gathers arbitrary token rows from a
//    bf16 copy of x (L2-resident at 4096 tokens) with tile::gather4 loads
//    (4 rows of 128 bytes each); the down GEMM's h rows are contiguous in slot
//    order and come with one 2D tile load per stage. Both land in the 128-byte
//    swizzled K-major layout and complete on a per-stage mbarrier.
//  * A (weights): the raw Q4_K bytes a stage needs (the 16-byte header and
//    two 16-byte quant chunks of each row's block) arrive by TMA through a 3D
//    byte map (16-byte chunk x chunk index x row); the Q6_K rows of a CTA are
//    one contiguous, 16-byte aligned slab (128 x 420 B) brought in by one bulk
//    copy. 8 warps dequantise (the reference's exact fp32 value rounded to
//    bf16; paired f32x2 arithmetic) into the same swizzled layout.
//  * one thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32) into TMEM;
//    tcgen05.commit arrives on the mbarriers that free the stage's buffers.
//  * warp-specialised: warp 0 produces (TMA), warp 1 issues the MMAs, warps
//    4..11 dequantise; the roles meet only on full/empty mbarrier rings, so
//    copies, dequantisation and tensor-core work of different stages overlap.
//  * epilogue (warps 4..11): tcgen05.ld of the accumulator (warp w reads TMEM
//    lanes 32*(w%4).. = its weight rows); up writes h = silu(g)*u as bf16 in
//    slot order, down adds w * y into out with fp32 reductions.
// No TMA load here uses cluster multicast. Every mbarrier wait is bounded: on
// timeout the kernel records an error flag, releases its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "moe.cuh"

namespace ofb {

constexpr int PF_M = 128;        // weight rows per CTA (MMA M)
constexpr int PF_NMAX = 256;     // token rows per tile (MMA N, max)
constexpr int PF_KS = 64;        // K elements per pipeline stage (= one 128-byte swizzle row)
constexpr int PF_NT = 384;       // threads per CTA: producer, MMA, 2 spare, 8 dequant/epilogue warps
constexpr int PF_DQ0 = 128;      // first dequantising thread
constexpr int PF_NDQW = 8;       // dequantising warps
constexpr int PF_STG = 3;        // ring depth for B and raw A
constexpr int PF_NA = 2;         // ring depth for dequantised A
constexpr int A_STAGE = PF_M * 128;        // 16 KB: 128 rows x 128 B
constexpr int B_STAGE = PF_NMAX * 128;     // 32 KB
constexpr int RAW4 = PF_M * 48;            // raw Q4_K bytes of one matrix per stage
constexpr long long WAIT_LIMIT = 1ll << 24;  // try_wait polls before giving up

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

// ---- copies -----------------------------------------------------------------
// TMA bulk copy global -> shared, completing on an mbarrier (no multicast).
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    mbar_expect_tx(bar, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Four 64-element rows (y0..y3, starting at column x) of a 2D bf16 tensor:
// 512 bytes, one-row box.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap *map, int x, int y0, int y1, int y2,
                                            int y3, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_u32(bar))
        : "memory");
}
// One 3D box at (c0, c1, c2).
__device__ __forceinline__ void tma_load3d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                           uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
// One 2D box (64 columns x 256 rows) at (x, y).
__device__ __forceinline__ void tma_tile2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ---- layout and conversion helpers ----------------------------------------------
// Byte offset of 16-byte chunk c of row r in a 128-byte swizzled K-major tile
// (1024-byte aligned base): the TMA/UMMA SWIZZLE_128B pattern.
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&p);
}
// Paired fp32 arithmetic (sm_100a f32x2): two elements per instruction.
__device__ __forceinline__ unsigned long long f2pack(float a, float b) {
    unsigned long long p;
    asm("mov.b64 %0, {%1,%2};" : "=l"(p) : "f"(a), "f"(b));
    return p;
}
__device__ __forceinline__ uint32_t f2_to_bf16(unsigned long long r) {
    float lo, hi;
    asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
    return pack_bf16(lo, hi);
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint32_t f2_fma_bf16(unsigned long long x, unsigned long long m, unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(m), "l"(c));
    return f2_to_bf16(r);
}
__device__ __forceinline__ uint32_t f2_mul_bf16(unsigned long long x, unsigned long long m) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(m));
    return f2_to_bf16(r);
}
// bytes (k, k+1) of w as the exact floats 2^23 + byte, as a pair
template <int K>
__device__ __forceinline__ unsigned long long byte_pair(uint32_t w) {
    return f2pack(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + K)),
                  __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541u + K)));
}
// 4 bytes at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_u32_2b(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(b[0], b[1], (unsigned)(a & 3) * 8);
}

// ---- A operand, Q4_K ----------------------------------------------------------------
// Raw bytes of one matrix for one stage, as three TMA boxes of 128 rows x 16
// bytes: [header | quant chunk 2c | quant chunk 2c+1] (chunk c of block b:
// elements 64c..64c+63, quant bytes 32c..32c+31).
__device__ __forceinline__ void q4_issue(const CUtensorMap *map, int row0, uint32_t dst, int stage, uint64_t *bar) {
    const int b = stage >> 2, c = stage & 3;
    tma_load3d(dst, map, 0, b * 9, row0, bar);
    tma_load3d(dst + 2048, map, 0, b * 9 + 1 + 2 * c, row0, bar);
    tma_load3d(dst + 4096, map, 0, b * 9 + 2 + 2 * c, row0, bar);
}

// Dequantising thread t (row r = t%128, half hh = t/128) writes chunks
// 4hh..4hh+3 of its row (low nibbles for hh = 0, high for hh = 1). Value =
// (d*sc)*q - dmin*m as one fused multiply-add: d*sc*q is exact in fp32
// (<= 21 significant bits), so the result equals the reference's two
// separately rounded operations.
__device__ __forceinline__ void q4_deq(const uint8_t *raw, int stage, int t, uint8_t *sa) {
    const int r = t & (PF_M - 1), hh = t >> 7, c = stage & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * 16);
    const uint4 qa = *reinterpret_cast<const uint4 *>(raw + 2048 + r * 16);
    const uint4 qb = *reinterpret_cast<const uint4 *>(raw + 4096 + r * 16);
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
        const uint32_t p0 = f2_fma_bf16(f2_add(byte_pair<0>(w0), nb2), d2, nm2);
        const uint32_t p1 = f2_fma_bf16(f2_add(byte_pair<2>(w0), nb2), d2, nm2);
        const uint32_t p2 = f2_fma_bf16(f2_add(byte_pair<0>(w1), nb2), d2, nm2);
        const uint32_t p3 = f2_fma_bf16(f2_add(byte_pair<2>(w1), nb2), d2, nm2);
        *reinterpret_cast<uint4 *>(sa + sw_off(r, 4 * hh + ch)) = make_uint4(p0, p1, p2, p3);
    }
}

// ---- A operand, Q6_K (from the raw slab in shared memory) ----------------------------
// 64-element chunk q of a block: half = q/2, quads 2*(q%2) and 2*(q%2)+1;
// thread t (row r, hh) writes quad 2*(q%2)+hh. Value = (d*sc)*(q-32), one
// rounding each, as the reference.
__device__ __forceinline__ void q6_deq(const uint8_t *slab, int row_bytes, int stage, int t, uint8_t *sa) {
    const int r = t & (PF_M - 1), hh = t >> 7;
    const int b = stage >> 2, q64 = stage & 3, half6 = q64 >> 1, quad = 2 * (q64 & 1) + hh;
    const uint8_t *blk = slab + r * row_bytes + b * Q6K_BYTES;
    const uint8_t *ql = blk + half6 * 64 + (quad & 1) * 32;
    const uint8_t *qh = blk + 128 + half6 * 32;
    const int si = 192 + half6 * 8 + quad * 2;
    const float d = half_bits_ref((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
    const float ds0 = __fmul_rn(d, (float)(int8_t)blk[si]), ds1 = __fmul_rn(d, (float)(int8_t)blk[si + 1]);
    const unsigned long long nb2 = f2pack(-8388640.0f, -8388640.0f);  // -(2^23 + 32)
    const int nsh = (quad >= 2) ? 4 : 0, hsh = 2 * quad;
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const float ds = ch < 2 ? ds0 : ds1;  // l = 8ch..8ch+7, scale index l/16
        const unsigned long long d2 = f2pack(ds, ds);
        uint32_t q[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
            const uint32_t wl = lds_u32_2b(ql + ch * 8 + h2 * 4), wh = lds_u32_2b(qh + ch * 8 + h2 * 4);
            q[h2] = ((wl >> nsh) & 0x0F0F0F0Fu) | (((wh >> hsh) & 0x03030303u) << 4);
        }
        const uint32_t p0 = f2_mul_bf16(f2_add(byte_pair<0>(q[0]), nb2), d2);
        const uint32_t p1 = f2_mul_bf16(f2_add(byte_pair<2>(q[0]), nb2), d2);
        const uint32_t p2 = f2_mul_bf16(f2_add(byte_pair<0>(q[1]), nb2), d2);
        const uint32_t p3 = f2_mul_bf16(f2_add(byte_pair<2>(q[1]), nb2), d2);
        *reinterpret_cast<uint4 *>(sa + sw_off(r, 4 * hh + ch)) = make_uint4(p0, p1, p2, p3);
    }
}

__device__ __forceinline__ int asg_token_p(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

// Parity of the phase that completes the n-th use (n = 0, 1, ...) of a ring
// slot is n & 1; a producer refilling a slot for use n >= 1 waits for the
// consumer's release of use n-1, parity (n-1) & 1.
struct Rings {
    uint64_t bfull[PF_STG], bempty[PF_STG];   // B: TMA -> MMA
    uint64_t rfull[PF_STG], rempty[PF_STG];   // raw A: TMA -> dequant
    uint64_t afull[PF_NA], aempty[PF_NA];     // bf16 A: dequant -> MMA
    uint64_t done;                            // all MMAs complete -> epilogue
};
__device__ __forceinline__ void rings_init(Rings &R) {
    for (int i = 0; i < PF_STG; i++) {
        mbar_init(&R.bfull[i], 1);
        mbar_init(&R.bempty[i], 1);
        mbar_init(&R.rfull[i], 1);
        mbar_init(&R.rempty[i], PF_NDQW);
    }
    for (int i = 0; i < PF_NA; i++) {
        mbar_init(&R.afull[i], PF_NDQW);
        mbar_init(&R.aempty[i], 1);
    }
    mbar_init(&R.done, 1);
}

// MMA role (one thread): per stage wait for A and B, issue the K = 64 slice
// of the product into each accumulator, release both buffers.
template <int NACC>
__device__ __forceinline__ bool mma_role(Rings &R, int nstages, const uint8_t *abf, const uint8_t *bst,
                                         uint32_t tbase, uint32_t idesc) {
    bool ok = true;
    for (int i = 0; i < nstages && ok; i++) {
        const int sa = i % PF_NA, sb = i % PF_STG;
        ok = mbar_wait(&R.afull[sa], (i / PF_NA) & 1) && mbar_wait(&R.bfull[sb], (i / PF_STG) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t aa = smem_u32(abf + sa * NACC * A_STAGE), bb = smem_u32(bst + sb * B_STAGE);
#pragma unroll
        for (int kk = 0; kk < PF_KS / 16; kk++) {
            const uint64_t bd = sw128_desc(bb + kk * 32);
#pragma unroll
            for (int m = 0; m < NACC; m++)
                mma_bf16(tbase + m * 256, sw128_desc(aa + m * A_STAGE + kk * 32), bd, idesc, (i | kk) != 0);
        }
        mma_commit(&R.aempty[sa]);
        mma_commit(&R.bempty[sb]);
    }
    mma_commit(&R.done);  // arrives once all issued MMAs complete
    return ok;
}

// ---- phase 1: gate/up ----------------------------------------------------------------
constexpr int UP_SMEM = 1024 + PF_STG * B_STAGE + PF_NA * 2 * A_STAGE + PF_STG * 2 * RAW4;

__global__ void __launch_bounds__(PF_NT, 1)
    prefill_up_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap umap,
                      const __grid_constant__ CUtensorMap gmap_sh, const __grid_constant__ CUtensorMap umap_sh) {
    extern __shared__ uint8_t psm_raw[];
    uint8_t *psm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Rings R;
    __shared__ uint32_t tslot;
    __shared__ int trow[PF_NMAX];
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int u = a.tile_slot[tile], s0 = a.tile_start[tile], n = a.tile_n[tile];
    const int e = a.slot_expert[u];
    const int m0 = blockIdx.y * PF_M;
    const int TK = a.T * a.K;
    // token row of each tile row; padding rows repeat the first token (their
    // accumulator columns are never read)
    for (int i = threadIdx.x; i < PF_NMAX; i += PF_NT)
        trow[i] = asg_token_p(a.assign[s0 + (i < n ? i : 0)], TK, a.K);
    if (threadIdx.x == 0) rings_init(R);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 512);  // gate: cols [0,256), up: [256,512); syncs the CTA

    uint8_t *bst = psm;                          // [PF_STG][B_STAGE]        1024-aligned
    uint8_t *abf = bst + PF_STG * B_STAGE;       // [PF_NA][gate A | up A]   1024-aligned
    uint8_t *raw = abf + PF_NA * 2 * A_STAGE;    // [PF_STG][gate raw | up raw]
    const int nn = (n + 15) & ~15;               // MMA N and rows fetched per stage
    const int nstages = a.D / PF_KS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = true;
    if (warp == 0) {
        // producer: B by gather4 (lanes split the nn/4 gathers), raw A by lane 0
        const CUtensorMap *gm = e == a.E ? &gmap_sh : &gmap, *um = e == a.E ? &umap_sh : &umap;
        const int row0 = (e == a.E ? 0 : e * a.H) + m0;
        for (int i = 0; i < nstages && ok; i++) {
            const int sb = i % PF_STG, use = i / PF_STG;
            if (use > 0) ok = mbar_wait(&R.bempty[sb], (use - 1) & 1);
            if (!ok) break;
            if (lane == 0) mbar_expect_tx(&R.bfull[sb], nn * 128);
            __syncwarp();
            const uint32_t dst = smem_u32(bst + sb * B_STAGE);
            for (int g = lane; g < nn / 4; g += 32)
                tma_gather4(dst + g * 512, &xmap, i * PF_KS, trow[4 * g], trow[4 * g + 1], trow[4 * g + 2],
                            trow[4 * g + 3], &R.bfull[sb]);
            if (use > 0) ok = mbar_wait(&R.rempty[sb], (use - 1) & 1);
            if (!ok) break;
            if (lane == 0) {
                mbar_expect_tx(&R.rfull[sb], 2 * RAW4);
                const uint32_t rd = smem_u32(raw + sb * 2 * RAW4);
                q4_issue(gm, row0, rd, i, &R.rfull[sb]);
                q4_issue(um, row0, rd + RAW4, i, &R.rfull[sb]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) ok = mma_role<2>(R, nstages, abf, bst, tbase, instr_desc(nn));
    } else if (warp >= PF_DQ0 / 32) {
        const int t = threadIdx.x - PF_DQ0;
        for (int i = 0; i < nstages && ok; i++) {
            const int sr = i % PF_STG, sa = i % PF_NA;
            ok = mbar_wait(&R.rfull[sr], (i / PF_STG) & 1);
            if (ok && i >= PF_NA) ok = mbar_wait(&R.aempty[sa], (i / PF_NA - 1) & 1);
            if (!ok) break;
            uint8_t *ag = abf + sa * 2 * A_STAGE;
            q4_deq(raw + sr * 2 * RAW4, i, t, ag);
            q4_deq(raw + sr * 2 * RAW4 + RAW4, i, t, ag + A_STAGE);
            async_proxy_fence();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&R.rempty[sr]);
                mbar_arrive(&R.afull[sa]);
            }
        }
        if (ok) ok = mbar_wait(&R.done, 0);
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else if (warp >= PF_DQ0 / 32) {
        // warp w reads TMEM lanes 32*(w%4).. (its rows), columns of half (w-4)/4
        const int q = warp & 3;
        const int m = m0 + q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int half = nn / 2, j_beg = ((warp - PF_DQ0 / 32) >> 2) * half;
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
// (128 x 420 B at H = 512): one bulk copy brings it in; stages copy only B.
__host__ __device__ inline int down_slab_bytes(int H) { return PF_M * (H / QK) * Q6K_BYTES; }
__host__ __device__ inline int down_smem(int H) {
    return 1024 + PF_STG * B_STAGE + PF_NA * A_STAGE + down_slab_bytes(H);
}

__global__ void __launch_bounds__(PF_NT, 1)
    prefill_down_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap hmap) {
    extern __shared__ uint8_t psm_raw[];
    uint8_t *psm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Rings R;
    __shared__ uint64_t slab_bar;
    __shared__ uint32_t tslot;
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
    uint8_t *bst = psm;                        // [PF_STG][B_STAGE]
    uint8_t *abf = bst + PF_STG * B_STAGE;     // [PF_NA][A_STAGE]
    uint8_t *slab = abf + PF_NA * A_STAGE;     // raw Q6_K rows (16-byte aligned)
    for (int i = threadIdx.x; i < n; i += PF_NT) {
        const int asg = a.assign[s0 + i];
        const int t = asg_token_p(asg, TK, a.K);
        tok[i] = t;
        wgt[i] = asg < TK ? a.w[asg] : (a.shared_gate ? a.gsc[t] : 1.0f);
    }
    if (threadIdx.x == 0) {
        rings_init(R);
        mbar_init(&slab_bar, 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t tbase = tmem_alloc(&tslot, 256);  // syncs the CTA

    const int nn = (n + 15) & ~15;
    const int nstages = a.H / PF_KS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = true;
    if (warp == 0) {
        // producer: the slab, then per stage one 64 x 256 box of h rows (rows
        // past the tile are not used; rows past the tensor read as zero and
        // still count toward the transaction bytes)
        if (lane == 0) {
            bulk_copy(slab, slab_src, down_slab_bytes(a.H), &slab_bar);
            for (int i = 0; i < nstages && ok; i++) {
                const int sb = i % PF_STG, use = i / PF_STG;
                if (use > 0) ok = mbar_wait(&R.bempty[sb], (use - 1) & 1);
                if (!ok) break;
                mbar_expect_tx(&R.bfull[sb], B_STAGE);
                tma_tile2d(smem_u32(bst + sb * B_STAGE), &hmap, i * PF_KS, s0, &R.bfull[sb]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) ok = mma_role<1>(R, nstages, abf, bst, tbase, instr_desc(nn));
    } else if (warp >= PF_DQ0 / 32) {
        const int t = threadIdx.x - PF_DQ0;
        ok = mbar_wait(&slab_bar, 0);
        for (int i = 0; i < nstages && ok; i++) {
            const int sa = i % PF_NA;
            if (i >= PF_NA) ok = mbar_wait(&R.aempty[sa], (i / PF_NA - 1) & 1);
            if (!ok) break;
            q6_deq(slab, row_bytes, i, t, abf + sa * A_STAGE);
            async_proxy_fence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&R.afull[sa]);
        }
        if (ok) ok = mbar_wait(&R.done, 0);
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
    } else if (warp >= PF_DQ0 / 32) {
        const int q = warp & 3;
        const int row = n0 + q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int half = nn / 2, j_beg = ((warp - PF_DQ0 / 32) >> 2) * half;
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

// Q4_K rows as a 3D byte tensor: 16-byte chunk x chunk index in the row x
// row; boxes of one chunk x 128 rows.
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
    const cuuint64_t dims[3] = {16, row_bytes / 16, rows};
    const cuuint64_t strides[2] = {16, row_bytes};
    const cuuint32_t box[3] = {16, 1, (cuuint32_t)PF_M};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (Q4_K rows) failed (%d)", (int)r);
        return OFB_ECUDA;
    }
    return OFB_OK;
}

int launch_prefill(const LayerArgs &la, const float *x, int *n_slots, __nv_bfloat16 *xb, __nv_bfloat16 *hb,
                   int *tiles, int *err, cudaStream_t s, cudaEvent_t before, cudaEvent_t between) {
    const int T = la.T, D = la.D, H = la.H;
    const int max_tiles = prefill_max_tiles(T, la.K, la.E);
    const int n_asg = T * la.K + T;
    int *n_tiles = tiles, *tile_slot = tiles + 1, *tile_start = tile_slot + max_tiles,
        *tile_n = tile_start + max_tiles;
    CUtensorMap xmap, hmap, gmap, umap, gmap_sh, umap_sh;
    int st;
    if ((st = encode_bf16_2d(&xmap, xb, D, T, 1))) return st;            // gather4 wants one-row boxes
    if ((st = encode_bf16_2d(&hmap, hb, H, n_asg, PF_NMAX))) return st;  // 64 x 256 boxes
    if ((st = encode_q4_rows(&gmap, la.gate, D, (uint64_t)la.E * H))) return st;
    if ((st = encode_q4_rows(&umap, la.up, D, (uint64_t)la.E * H))) return st;
    if (la.has_shared) {
        if ((st = encode_q4_rows(&gmap_sh, la.gate_sh, D, H))) return st;
        if ((st = encode_q4_rows(&umap_sh, la.up_sh, D, H))) return st;
    } else {
        gmap_sh = gmap;  // never read: no slot names the shared expert
        umap_sh = umap;
    }
    to_bf16_kernel<<<grid_for((size_t)T * D / 4, 256, 148 * 8), 256, 0, s>>>(x, (size_t)T * D, xb);
    tile_plan_kernel<<<1, 256, 0, s>>>(n_slots, la.slot_start, n_tiles, tile_slot, tile_start, tile_n);
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
    prefill_up_kernel<<<dim3(max_tiles, H / PF_M), PF_NT, smem_up, s>>>(a, xmap, gmap, umap, gmap_sh, umap_sh);
    if (between) cudaEventRecord(between, s);
    prefill_down_kernel<<<dim3(max_tiles, D / PF_M), PF_NT, smem_dn, s>>>(a, hmap);
    OFB_CHECK_LAUNCH("prefill kernels");
    return OFB_OK;
}

}  // namespace ofb
