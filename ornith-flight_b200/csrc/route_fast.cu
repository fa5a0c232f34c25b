// route_fast.cu — certified routing for decode-sized batches, in two PDL
// kernels: router rows (logits + error bounds, shared-expert gates, the
// activation quantisation for the decode expert kernels) and per-token
// selection (top-k, certificate, weights) plus the dispatch plan.
//
// The reference's router logit is a sequential fp32 sum with separate
// multiply and add (engine/src/model.c:1019-1025). Reproducing it literally
// costs a 2048-long dependent add chain per (token, expert): ~4 us of pure
// latency at decode. Instead:
//  1. One warp per (token, router row) computes L~ = sum_d x_d w_d in fp64
//     (products exact, 64-term lane segments, warp scan of segment sums)
//     together with a rigorous bound B on |L_ref - L~|, where L_ref is the
//     reference's sequentially rounded fp32 value:
//       L_ref - sum p_i = sum (fl(p_i) - p_i) + sum (rounding of add i),
//       |fl(p_i) - p_i| <= u|p_i|, |rounding of add i| <= u|s_i|,
//       sum_i |s_i| <= sum_i |P_i| + n*gamma_n*A     (P_i exact prefixes),
//     so B = u*(A + S_P + n*gamma_n*A), A = sum|p_i|, S_P an upper bound of
//     sum|P_i| from the segment scan (u = 2^-24, gamma_n = nu/(1-nu)),
//     inflated by 2^-9 relative plus 2^-60 absolute for the fp64 arithmetic.
//  2. One block per token ranks the experts by L~ (warp bitonic sorts, then a
//     rank among the per-warp winners) and CERTIFIES the reference's top-k:
//     every adjacent gap in the top-k and the gap to every other expert must
//     exceed the two bounds plus a margin M = 2^-14, large enough that
//     expf(l - max) and the divided probabilities stay strictly ordered after
//     fp32 rounding. Then the reference's exchange sort (model.c:1042-1049),
//     which only swaps on strict '>', yields exactly this order: the indices
//     are bit-exact.
//  3. Otherwise (two logits closer than ~1e-4) the block recomputes the
//     uncertain candidates with the reference's exact sequential chain and the
//     host library's expf (exact_expf.h), and emulates the exchange sort on
//     them; if two candidate probabilities could round together, it
//     recomputes every expert exactly (bit-exact softmax sum) before sorting.
// Routing weights come from fp32 softmax of L~ (or the exact logits where
// computed): within ~1e-6 relative of the reference's (bit-exact in the
// full-recompute case). The block finishing the last token builds the plan.
// Both kernels are launched with programmatic dependent launch: the row
// kernel loads its router rows before waiting for the previous kernel in the
// stream, so the router read overlaps the previous layer's tail.
// Interleaved-layout routers and large batches use the exact kernels of
// route.cu.
#include "common.cuh"
#include "exact_expf.h"
#include "moe.cuh"
#include "route.cuh"
#include "exchange.cuh"
#include "exact_route.cuh"
#include "plan.cuh"

namespace ofb {

DTRACE_DEFINE(rf)

// Optional per-block timeline of route_select_fast (build with
// -DOFB_RS_TRACE): globaltimer at each step of the last launch, one row per
// token block, read back with ofb_debug_rs_trace.
#ifdef OFB_RS_TRACE
__device__ unsigned long long g_rs_tr[64][16];
#define RS_MARK(i) \
    if (threadIdx.x == 0 && blockIdx.x < 64) { unsigned long long t_; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); g_rs_tr[blockIdx.x][i] = t_; }
extern "C" int ofb_debug_rs_trace(unsigned long long *host) {
    return cudaMemcpyFromSymbol(host, g_rs_tr, sizeof(g_rs_tr)) == cudaSuccess ? 0 : 1;
}
#else
#define RS_MARK(i)
#endif

constexpr int RR_WARPS = 8;  // router rows per block in the row kernel (at most)
constexpr int FR_WARPS = 8;
constexpr int FR_THREADS = FR_WARPS * 32;
constexpr double FR_MARGIN = 0x1.0p-14;
constexpr int FW_PER_LANE = 8;  // warp top-k path: experts per lane (E <= 256)

struct FastRouteArgs {
    const float *W, *x, *gate_v;
    int T, D, E, K, routing, renorm;
    double bound_scale;  // (1 + 2^-9) * u, u = 2^-24
    double ngam;         // n * gamma_n
    double2 *cand;       // [T][E]: (L~, B)
    int *all_cnt;        // [1], zero between calls
    int *stats;          // [3]: certified, candidate recompute, full recompute
    uint32_t *idx;
    float *w, *gsc;
    unsigned char *xq;  // [T][xq_stride(D)] quantised activations, or NULL
    PlanArgs plan;
    const int *flagged;    // large batches: tokens the warp certificate left (or NULL)
    const int *n_flagged;
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Quantised activations of 32-element sub-block sb (one warp):
// x ~= s * (256*xh + xl), xh int8, xl uint8, s = max|x|/32767; plus sum(x).
__device__ __forceinline__ void quantize_subblock(float v, unsigned char *q, int D, int sb, int lane) {
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m / 32767.0f;
    const int xi = (m > 0.0f) ? __float2int_rn(v / s) : 0;
    q[sb * 32 + lane] = (unsigned char)(xi >> 8);       // floor(xi / 256), int8
    q[D + sb * 32 + lane] = (unsigned char)(xi & 255);  // remainder, uint8
    const float xsum = warp_sum(v);
    if (lane == 0) {
        reinterpret_cast<float *>(q + 2 * D)[sb] = s;
        reinterpret_cast<float *>(q + 2 * D)[D / 32 + sb] = xsum;
    }
}

// ---- kernel 1: router rows ---------------------------------------------------
// Lane l of a row's warp owns the contiguous segment [l*seg, (l+1)*seg),
// seg = D/32 (the prefix bound below needs contiguous segments). Reading such
// segments straight from global memory makes every 16-byte load of a warp
// touch 32 sectors, so the block first moves its router rows (before the
// dependent-launch wait: the router is static) and the token's x (after it)
// into shared memory with coalesced loads, in a segment-major layout padded
// by 4 floats per segment (a quarter-warp's 16-byte reads hit distinct banks).
__host__ __device__ inline int rr_seg_ld(int D) { return D / 32 + 4; }  // floats per lane segment
__host__ __device__ inline size_t rr_smem(int D, int nw) { return (size_t)(nw + 1) * 32 * rr_seg_ld(D) * 4; }

// Coalesced copy of n floats (n a multiple of 4) into the segment-major layout.
__device__ __forceinline__ void rr_stage(float *dst, const float *__restrict__ src, int D, int i0, int step) {
    const int seg = D / 32, ld = rr_seg_ld(D);
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll 4
    for (int q = i0; q < D / 4; q += step) {
        const int e = 4 * q, l = e / seg;
        *reinterpret_cast<float4 *>(dst + l * ld + (e - l * seg)) = __ldg(s4 + q);
    }
}

__global__ void __launch_bounds__(RR_WARPS * 32) route_rows_kernel(FastRouteArgs a) {
    DTRACE_START(rf, 0)
    pdl_trigger();
    extern __shared__ __align__(16) float rr_sm[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int t = blockIdx.y;
    const int E = a.E, D = a.D, ld = rr_seg_ld(D);
    const int r = blockIdx.x * nw + wid;  // router row; r == E is the gate vector
    const float *xt = a.x + (size_t)t * D;
    const bool has_row = (r < E) || (r == E && a.gate_v);
    const int seg = D / 32;  // multiple of 8
    float *xs = rr_sm, *wrow = rr_sm + (size_t)(1 + wid) * 32 * ld;
    // the router is static: stage it before waiting for the producer of x
    if (has_row) rr_stage(wrow, (r < E) ? a.W + (size_t)r * D : a.gate_v, D, lane, 32);
    pdl_wait();
    DTRACE_WAITED(rf, 0)
    rr_stage(xs, xt, D, threadIdx.x, blockDim.x);
    if (a.xq && r > E) {
        // warps past the router rows and the gate vector quantise x, beside
        // the rows rather than in front of them
        unsigned char *q = a.xq + (size_t)t * xq_stride(D);
        const int nq = gridDim.x * nw - (E + 1);
        for (int sb = r - (E + 1); sb < D / 32; sb += nq)
            quantize_subblock(__ldg(xt + sb * 32 + lane), q, D, sb, lane);
    }
    __syncthreads();
    if (!has_row) {
        DTRACE_END(rf, 0)
        return;
    }
    const float4 *w4 = reinterpret_cast<const float4 *>(wrow + lane * ld);
    const float4 *x4 = reinterpret_cast<const float4 *>(xs + lane * ld);
    double P = 0.0, SP = 0.0, A = 0.0;
#pragma unroll 4
    for (int j = 0; j < seg / 4; j++) {
        const float4 wv = w4[j], xv = x4[j];
        const double p0 = (double)xv.x * wv.x, p1 = (double)xv.y * wv.y;
        const double p2 = (double)xv.z * wv.z, p3 = (double)xv.w * wv.w;
        P += p0; SP += fabs(P);
        P += p1; SP += fabs(P);
        P += p2; SP += fabs(P);
        P += p3; SP += fabs(P);
        A += (fabs(p0) + fabs(p1)) + (fabs(p2) + fabs(p3));
    }
    // exclusive scan of segment sums -> |prefix| bound of this segment
    double inc = P;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double up = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += up;
    }
    const double sp_bound = (double)seg * fabs(inc - P) + SP;
    const double L = warp_sum_d(P);
    const double SPt = warp_sum_d(sp_bound);
    const double At = warp_sum_d(A);
    if (lane == 0) {
        if (r < E)
            a.cand[(size_t)t * E + r] = make_double2(L, a.bound_scale * (At + SPt + a.ngam * At) + 0x1.0p-60);
        else
            a.gsc[t] = 1.0f / (1.0f + expf(-(float)L));
    }
    DTRACE_END(rf, 0)
}

// ---- kernel 2: selection, one block per token ---------------------------------
struct KeyIdx { float k; int i; };
__device__ __forceinline__ bool better(KeyIdx a, KeyIdx b) { return a.k > b.k || (a.k == b.k && a.i < b.i); }

// Descending bitonic sort of one value per lane (lane 0 ends with the best).
__device__ __forceinline__ KeyIdx warp_sort_desc(KeyIdx v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            KeyIdx o;
            o.k = __shfl_xor_sync(0xffffffffu, v.k, j);
            o.i = __shfl_xor_sync(0xffffffffu, v.i, j);
            const bool keep_better = (((lane & j) == 0) == ((lane & k) == 0));
            if (keep_better ? better(o, v) : better(v, o)) v = o;
        }
    }
    return v;
}

__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float r = 0.f;
    for (int i = 0; i < FR_WARPS; i++) r += red[i];
    return r;
}

// Per-warp scratch of the certified selection (top_k <= 16).
struct WarpSel { int top[16]; double L[16], B[16]; float w[16]; };

// Certified top-k of token t by one warp (E <= 32 * FW_PER_LANE): K rounds of
// a warp argmax on order-preserving 32-bit keys of float(L~) (a mis-order
// between logits that round to the same float cannot pass the certificate,
// which checks every adjacent gap on the double values), then the
// certificate, then - when it holds - the weights (fp32 softmax of L~,
// model.c:1027-1049 / :300-316 forms) written to idx / w. Ls / Bs, when
// given, receive every (L~, B) of the token for a block fallback.
__device__ bool certify_token_warp(const FastRouteArgs &a, int t, WarpSel &ws, double *Ls, double *Bs) {
    const int lane = threadIdx.x & 31, E = a.E, K = a.K;
    const double2 *cd = a.cand + (size_t)t * E;
    double L[FW_PER_LANE], B[FW_PER_LANE];
    uint32_t key[FW_PER_LANE];
    bool top[FW_PER_LANE];
#pragma unroll
    for (int j = 0; j < FW_PER_LANE; j++) {
        const int e = lane + 32 * j;
        top[j] = false;
        L[j] = -INFINITY;
        B[j] = 0.0;
        if (e < E) {
            const double2 v = cd[e];
            L[j] = v.x;
            B[j] = v.y;
            if (Ls) {
                Ls[e] = v.x;
                Bs[e] = v.y;
            }
        }
        const uint32_t u = __float_as_uint((float)L[j]);
        key[j] = (e < E) ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;
    }
    for (int q = 0; q < K; q++) {
        uint32_t lb = 0;
        int le = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < FW_PER_LANE; j++)
            if (!top[j] && key[j] > lb) {  // strict: the smallest index wins a tie
                lb = key[j];
                le = lane + 32 * j;
            }
        const uint32_t wb = __reduce_max_sync(0xffffffffu, lb);
        const int bi = (int)__reduce_min_sync(0xffffffffu, lb == wb ? (uint32_t)le : 0x7fffffffu);
#pragma unroll
        for (int j = 0; j < FW_PER_LANE; j++)
            if (lane + 32 * j == bi) {
                top[j] = true;
                ws.L[q] = L[j];
                ws.B[q] = B[j];
            }
        if (lane == 0) ws.top[q] = bi;
    }
    // certificate: adjacent gaps in the top-k, the last against the rest
    double hi_rest = -INFINITY;
#pragma unroll
    for (int j = 0; j < FW_PER_LANE; j++)
        if (lane + 32 * j < E && !top[j]) hi_rest = fmax(hi_rest, L[j] + B[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) hi_rest = fmax(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, o));
    __syncwarp();
    bool ok = true;
    if (lane < K) {
        const double nxt = lane + 1 < K ? ws.L[lane + 1] + ws.B[lane + 1] : hi_rest;
        ok = ws.L[lane] - ws.B[lane] > nxt + FR_MARGIN;
        if (lane == K - 1) ok = ok && (ws.L[lane] - ws.L[0] > -80.0);
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) return false;
    const float m = (float)ws.L[0];
    float sum = 0.f;
    if (a.routing == OFB_ROUTE_FORWARD) {
#pragma unroll
        for (int j = 0; j < FW_PER_LANE; j++)
            if (lane + 32 * j < E) sum += expf((float)L[j] - m);
    } else if (lane < K) {
        sum = expf((float)ws.L[lane] - m);
    }
    sum = warp_sum(sum);
    float wq = 0.f;
    if (lane < K) wq = expf((float)ws.L[lane] - m) / sum;
    if (lane < K) ws.w[lane] = wq;
    __syncwarp();
    if (lane < K) {
        float ss = 0.f;
        for (int q = 0; q < K; q++) ss += ws.w[q];
        if (a.routing == OFB_ROUTE_FORWARD && a.renorm) wq = wq / ss;
        a.idx[(size_t)t * K + lane] = (uint32_t)ws.top[lane];
        a.w[(size_t)t * K + lane] = wq;
    }
    __syncwarp();
    if (lane < K) ws.w[lane] = wq;
    if (lane == 0 && a.stats) atomicAdd(&a.stats[0], 1);
    __syncwarp();
    return true;
}

// The dispatch plan of one token (what build_plan makes for T = 1): kept
// experts in ascending id order, then the shared slot. One warp.
__device__ void one_token_plan(const FastRouteArgs &a, const WarpSel &ws) {
    const int lane = threadIdx.x & 31, K = a.K;
    const bool kept = lane < K && !(ws.w[lane] < 1e-6f);
    const unsigned km = __ballot_sync(0xffffffffu, kept);
    const int eq = lane < K ? ws.top[lane] : 0;
    int rank = 0;
    for (int q = 0; q < K; q++) rank += ((km >> q) & 1) && ws.top[q] < eq;
    const PlanArgs &p = a.plan;
    if (kept) {
        p.slot_expert[rank] = eq;
        p.slot_start[rank] = rank;
        p.assign[rank] = lane;
    }
    if (lane == 0) {
        const int nk = __popc(km);
        if (p.has_shared) {
            p.slot_expert[nk] = a.E;
            p.slot_start[nk] = nk;
            p.slot_start[nk + 1] = nk + 1;
            p.assign[nk] = K;
            *p.n_slots = nk + 1;
        } else {
            p.slot_start[nk] = nk;
            *p.n_slots = nk;
        }
    }
}

// Large batches: one warp per token; tokens whose certificate fails go to the
// flagged list for the warp fallback (route_fallback_warps).
__global__ void __launch_bounds__(256) route_certify_warps(FastRouteArgs a, int *flagged, int *n_flagged) {
    __shared__ WarpSel sel[8];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + wid;
    if (t >= a.T) return;
    const bool ok = certify_token_warp(a, t, sel[wid], nullptr, nullptr);
    if (!ok && lane == 0) flagged[atomicAdd(n_flagged, 1)] = t;
    if (a.gate_v && a.gsc) {
        // the token's shared-expert gate sigmoid(x . v), as shared_gate_kernel
        // computes it (same order), while this warp has the token
        const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.D);
        const float4 *v4 = reinterpret_cast<const float4 *>(a.gate_v);
        float z = 0.f;
        for (int i = lane; i < a.D / 4; i += 32) {
            const float4 p = __ldg(x4 + i), q = __ldg(v4 + i);
            z += p.x * q.x + p.y * q.y + p.z * q.z + p.w * q.w;
        }
        z = warp_sum(z);
        if (lane == 0) a.gsc[t] = 1.0f / (1.0f + expf(-z));
    }
}

// ---- large batches: the tokens the warp certificate left, one warp each ----
// The block fallback of route_select_fast restated at warp granularity, so
// that every flagged token of a batch runs at once: top-k of float(L~) (ties
// to the smaller index), candidates = experts with L~ + B >= min over the
// top-k of (L~ - B) - margin in ascending expert order, their exact logits
// (lane c runs candidate c's reference-order chain, exact_logit's
// arithmetic, its router row streamed through shared memory by cp.async), the
// reference's selection over the candidates (exchange_pass), weights from L~.
// Forward routing whose candidate probabilities come within a few ulps
// recomputes every logit and the reference's softmax exactly.
constexpr int FB_WARPS = 2;                  // tokens per block (two blocks fit an SM)
constexpr int FB_CK = XL_CK, FB_LD = XL_LD;  // chain chunk (floats) and padded lane stride
constexpr int FB_ST = 4;                      // chunks in flight per lane

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__host__ __device__ inline size_t fb_warp_smem(int E, int D) {
    return ((size_t)FB_ST * 32 * FB_LD * 4 + (size_t)D * 4 + (size_t)E * 6 * 4 + 15) & ~(size_t)15;
}

__global__ void __launch_bounds__(FB_WARPS * 32) route_fallback_warps(FastRouteArgs a) {
    extern __shared__ __align__(16) unsigned char fb_sm[];
    __shared__ WarpSel sel[FB_WARPS];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.E, D = a.D, K = a.K;
    unsigned char *mine = fb_sm + wid * fb_warp_smem(E, D);
    float *slots = reinterpret_cast<float *>(mine) + lane * FB_LD;    // this lane's chunk slots
    float *xs = reinterpret_cast<float *>(mine) + FB_ST * 32 * FB_LD;  // [D]
    float *Lf = xs + D;                                                // [E] float(L~)
    int *clist = reinterpret_cast<int *>(Lf + E);                      // [E] candidates
    float *cv = reinterpret_cast<float *>(clist + E);                  // [E] their values
    int *cid = reinterpret_cast<int *>(cv + E);                        // [E]
    float *cov = reinterpret_cast<float *>(cid + E);                   // [E] exchange scratch
    int *coid = reinterpret_cast<int *>(cov + E);                      // [E]
    const int n_tok = *a.n_flagged;
    for (int it = blockIdx.x * FB_WARPS + wid; it < n_tok; it += gridDim.x * FB_WARPS) {
        const int t = a.flagged[it];
        WarpSel &ws = sel[wid];
        certify_token_warp(a, t, ws, nullptr, nullptr);  // top-k only: the token failed it before
        const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)t * D);
        for (int d = lane; d < D / 4; d += 32) reinterpret_cast<float4 *>(xs)[d] = x4[d];
        double lo_min = INFINITY;
        for (int q = 0; q < K; q++) lo_min = fmin(lo_min, ws.L[q] - ws.B[q]);
        // candidates in ascending expert order
        const double2 *cd = a.cand + (size_t)t * E;
        int nc = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            bool cand = false;
            if (e < E) {
                const double2 v = cd[e];
                Lf[e] = (float)v.x;
                cand = v.x + v.y >= lo_min - FR_MARGIN;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, cand);
            if (cand) clist[nc + __popc(bal & ((1u << lane) - 1u))] = e;
            nc += __popc(bal);
        }
        __syncwarp();
        for (int c0 = 0; c0 < nc; c0 += 32) {
            const int c = c0 + lane;
            if (c < nc) {
                const int e = clist[c];
                cv[c] = exact_logit_lane<FB_ST>(a.W + (size_t)e * D, xs, D, slots);
                cid[c] = e;
            }
        }
        __syncwarp();
        int mode = 1;
        if (a.routing == OFB_ROUTE_FORWARD) {
            // probabilities are ordered like expf(l - max) unless two of them
            // are within a few ulps (then the division could tie them)
            float m = -INFINITY;
            for (int c = lane; c < nc; c += 32) m = fmaxf(m, cv[c]);
            m = warp_max(m);
            for (int c = lane; c < nc; c += 32) cv[c] = ofb_exact_expf(__fsub_rn(cv[c], m));
            __syncwarp();
            bool close = false;
            for (int c = lane; c < nc; c += 32)
                for (int c2 = 0; c2 < nc; c2++)
                    if (c2 != c && close_ulps(cv[c], cv[c2], 4)) close = true;
            if (__any_sync(0xffffffffu, close)) {
                // ---- every logit exact, the reference's softmax
                mode = 2;
                for (int e0 = 0; e0 < E; e0 += 32) {
                    const int e = e0 + lane;
                    if (e < E) {
                        cv[e] = exact_logit_lane<FB_ST>(a.W + (size_t)e * D, xs, D, slots);
                        cid[e] = e;
                    }
                }
                __syncwarp();
                float mx = -INFINITY;
                for (int e = lane; e < E; e += 32) mx = fmaxf(mx, cv[e]);
                mx = warp_max(mx);
                for (int e = lane; e < E; e += 32) cv[e] = ofb_exact_expf(__fsub_rn(cv[e], mx));
                __syncwarp();
                float sum = 0.0f;
                if (lane == 0)
                    for (int e = 0; e < E; e++) sum = __fadd_rn(sum, cv[e]);
                sum = __shfl_sync(0xffffffffu, sum, 0);
                for (int e = lane; e < E; e += 32) cv[e] = __fdiv_rn(cv[e], sum);
                __syncwarp();
                nc = E;
            }
        }
        exchange_topk(cv, cid, cov, coid, nc, K, lane);
        uint32_t *io = a.idx + (size_t)t * K;
        float *wo = a.w + (size_t)t * K;
        if (mode == 2) {
            // bit-exact: cv holds the reference's probabilities in its order
            if (lane == 0) {
                float ssum = 0.0f;
                for (int q = 0; q < K; q++) ssum = __fadd_rn(ssum, cv[q]);
                for (int q = 0; q < K; q++) {
                    io[q] = (uint32_t)cid[q];
                    wo[q] = a.renorm ? __fdiv_rn(cv[q], ssum) : cv[q];
                }
            }
        } else {
            const float m = Lf[cid[0]];
            float sum = 0.f;
            if (a.routing == OFB_ROUTE_FORWARD) {
                for (int e = lane; e < E; e += 32) sum += expf(Lf[e] - m);
            } else if (lane < K) {
                sum = expf(Lf[cid[lane]] - m);
            }
            sum = warp_sum(sum);
            float wq = lane < K ? expf(Lf[cid[lane]] - m) / sum : 0.f;
            float ss = 0.f;
            for (int q = 0; q < K; q++) ss += __shfl_sync(0xffffffffu, wq, q);
            if (lane < K) {
                io[lane] = (uint32_t)cid[lane];
                wo[lane] = (a.routing == OFB_ROUTE_FORWARD && a.renorm) ? wq / ss : wq;
            }
        }
        if (lane == 0 && a.stats) atomicAdd(&a.stats[mode], 1);
        __syncwarp();  // the next token reuses this warp's arrays
    }
}

// Dynamic shared memory of route_select_fast: Ls, Bs (f64), val, id, oval,
// oid, xs, taken, then (16-byte aligned) the exact-chain chunk buffers.
__host__ __device__ inline size_t xl_offset(int E, int D) {
    return ((size_t)E * (8 + 8 + 4 + 4 + 4 + 4 + 4) + (size_t)D * 4 + 15) & ~(size_t)15;
}
constexpr int FR_SMEM_MAX = 160 * 1024;

__global__ void __launch_bounds__(FR_THREADS) route_select_fast(FastRouteArgs a) {
    DTRACE_START(rf, 1)
    pdl_trigger();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, tid = threadIdx.x;
    const int E = a.E, D = a.D, K = a.K;

    extern __shared__ __align__(16) unsigned char smem[];
    double *Ls = reinterpret_cast<double *>(smem);     // [E]
    double *Bs = Ls + E;                                // [E]
    float *val = reinterpret_cast<float *>(Bs + E);     // [E]
    int *id = reinterpret_cast<int *>(val + E);         // [E]
    float *oval = reinterpret_cast<float *>(id + E);    // [E]
    int *oid = reinterpret_cast<int *>(oval + E);       // [E]
    float *xs = reinterpret_cast<float *>(oid + E);     // [D]
    int *taken = reinterpret_cast<int *>(xs + D);       // [E]
    float *wbuf = reinterpret_cast<float *>(smem + xl_offset(E, D));  // exact-chain chunk buffers
    __shared__ KeyIdx s_cand[32 * 17];
    __shared__ int s_top[17];
    __shared__ int s_mode;  // 0 certified, 1 candidate recompute, 2 full recompute
    __shared__ float s_red[FR_WARPS];
    __shared__ double s_hred[FR_WARPS];
    __shared__ float s_w[16];
    __shared__ int s_last;
    __shared__ WarpSel sel;
    // fallback: candidate experts in expert order, their values, sort scratch
    __shared__ int s_clist[1024], s_cid[1024], s_coid[1024];
    __shared__ float s_cv[1024], s_cov[1024];
    __shared__ int s_nc, s_full, s_wcnt[FR_WARPS];

    RS_MARK(0)
    pdl_wait();
    DTRACE_WAITED(rf, 1)
    RS_MARK(1)
    // one token per block
    {
    const int t = blockIdx.x;
    const float *xt = a.x + (size_t)t * D;
    const double2 *cd = a.cand + (size_t)t * E;
    if (E <= 32 * FW_PER_LANE) {
        // ---- warp 0: top-k, certificate and (when certified) weights from
        // registers; the block steps below run only for uncertain tokens
        if (wid == 0) {
            const bool ok = certify_token_warp(a, t, sel, Ls, Bs);
            if (lane == 0) s_mode = ok ? 0 : 1;
            if (lane < K) s_top[lane] = sel.top[lane];
            if (ok && a.T == 1 && a.plan.n_slots) one_token_plan(a, sel);
        }
        __syncthreads();
        if (s_mode == 0 && a.T == 1) {
            DTRACE_END(rf, 1)
            return;
        }
    } else {
    for (int e = tid; e < E; e += FR_THREADS) {
        const double2 v = cd[e];
        Ls[e] = v.x;
        Bs[e] = v.y;
        taken[e] = 0;
    }
    if (tid == 0) s_mode = 0;
    __syncthreads();
    // top K+1 by L~ (ties by index): per-32 chunk bitonic sort, then rank
    // the chunk winners. Ranking key is float; the certificate uses L~, B.
    const int kk = K < E ? K + 1 : K;
    const int nchunks = (E + 31) / 32;
    for (int c = wid; c < nchunks; c += FR_WARPS) {
        const int e = c * 32 + lane;
        KeyIdx v = (e < E) ? KeyIdx{(float)Ls[e], e} : KeyIdx{-INFINITY, 0x7fffffff};
        v = warp_sort_desc(v, lane);
        if (lane < kk) s_cand[c * kk + lane] = v;
    }
    __syncthreads();
    const int ncand = nchunks * kk;
    for (int i = tid; i < ncand; i += FR_THREADS) {
        const KeyIdx v = s_cand[i];
        int rank = 0;
        for (int j = 0; j < ncand; j++) rank += better(s_cand[j], v);
        if (rank < kk && v.i < E) s_top[rank] = v.i;
    }
    __syncthreads();
    if (tid < K) taken[s_top[tid]] = 1;
    __syncthreads();
    // certificate: adjacent gaps inside the top-k, and top-k vs the rest
    double hi_rest = -INFINITY;
    for (int e = tid; e < E; e += FR_THREADS)
        if (!taken[e]) hi_rest = fmax(hi_rest, Ls[e] + Bs[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) hi_rest = fmax(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, o));
    if (lane == 0) s_hred[wid] = hi_rest;
    __syncthreads();
    if (tid < K) {
        const int e0 = s_top[tid];
        double nxt;
        if (tid + 1 < K) {
            const int e1 = s_top[tid + 1];
            nxt = Ls[e1] + Bs[e1];
        } else {
            nxt = -INFINITY;
            for (int i = 0; i < FR_WARPS; i++) nxt = fmax(nxt, s_hred[i]);
        }
        bool ok = Ls[e0] - Bs[e0] > nxt + FR_MARGIN;
        if (tid == K - 1) ok = ok && (Ls[e0] - Ls[s_top[0]] > -80.0);
        if (!ok) s_mode = 1;
    }
    __syncthreads();
    }
    const bool warp_done = (E <= 32 * FW_PER_LANE) && s_mode == 0;  // weights already written
    RS_MARK(2)

    if (s_mode != 0) {
        // ---- candidate recompute with the reference's exact chain --------
        for (int d = tid; d < D; d += FR_THREADS) xs[d] = xt[d];
        double lo_min = INFINITY;
        for (int q = 0; q < K; q++) lo_min = fmin(lo_min, Ls[s_top[q]] - Bs[s_top[q]]);
        __syncthreads();
        // candidates in ascending expert order (a ballot prefix per round of
        // 256 experts): their exact chains occupy the first threads, and the
        // exchange sort runs over them alone - experts outside the list hold
        // -inf, never win a strict comparison, and so leave the candidates'
        // relative order as the full sort would.
        if (tid == 0) s_nc = 0;
        __syncthreads();
        for (int e0 = 0; e0 < E; e0 += FR_THREADS) {
            const int e = e0 + tid;
            const bool cand = e < E && (Ls[e] + Bs[e] >= lo_min - FR_MARGIN);
            if (e < E) {
                val[e] = -INFINITY;
                id[e] = e;
                taken[e] = cand;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, cand);
            if (lane == 0) s_wcnt[wid] = __popc(bal);
            __syncthreads();
            int off = s_nc;
            for (int q = 0; q < wid; q++) off += s_wcnt[q];
            if (cand) s_clist[off + __popc(bal & ((1u << lane) - 1u))] = e;
            __syncthreads();
            if (tid == 0)
                for (int q = 0; q < FR_WARPS; q++) s_nc += s_wcnt[q];
            __syncthreads();
        }
        const int nc = s_nc;
        RS_MARK(5)
#ifdef OFB_RS_TRACE
        if (tid == 0 && blockIdx.x < 64) g_rs_tr[blockIdx.x][11] = (unsigned long long)nc;
#endif
        exact_logits_block(a.W, D, xs, s_clist, nc, s_cv, wbuf, tid, FR_THREADS);
        __syncthreads();
        RS_MARK(6)
        for (int c = tid; c < nc; c += FR_THREADS) {
            const int e = s_clist[c];
            val[e] = s_cv[c];
            s_cid[c] = e;
        }
        if (tid == 0) s_full = 0;
        __syncthreads();
        if (a.routing == OFB_ROUTE_FORWARD) {
            // probabilities are ordered like expf(l - max) unless two of them
            // are within a few ulps (then the division could tie them)
            __shared__ float s_max;
            if (wid == 0) {
                float m = -INFINITY;
                for (int c = lane; c < nc; c += 32) m = fmaxf(m, s_cv[c]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (lane == 0) s_max = m;
            }
            __syncthreads();
            for (int c = tid; c < nc; c += FR_THREADS) s_cv[c] = ofb_exact_expf(__fsub_rn(s_cv[c], s_max));
            __syncthreads();
            for (int c = tid; c < nc; c += FR_THREADS)
                for (int c2 = 0; c2 < nc; c2++)
                    if (c2 != c && close_ulps(s_cv[c], s_cv[c2], 4)) s_full = 1;
            __syncthreads();
            if (s_full) {
                // ---- full recompute: every logit exact, softmax as the reference
                for (int e = tid; e < E; e += FR_THREADS)
                    val[e] = taken[e] ? val[e] : exact_logit(a.W + (size_t)e * D, xs, D);
                __syncthreads();
                if (tid == 0) {
                    float m = val[0];
                    for (int e = 1; e < E; e++) if (val[e] > m) m = val[e];
                    s_max = m;
                }
                __syncthreads();
                for (int e = tid; e < E; e += FR_THREADS) val[e] = ofb_exact_expf(__fsub_rn(val[e], s_max));
                __syncthreads();
                __shared__ float s_sum;
                if (tid == 0) {
                    float s = 0.0f;
                    for (int e = 0; e < E; e++) s = __fadd_rn(s, val[e]);
                    s_sum = s;
                    s_mode = 2;
                }
                __syncthreads();
                for (int e = tid; e < E; e += FR_THREADS) val[e] = __fdiv_rn(val[e], s_sum);
                __syncthreads();
            }
        }
        RS_MARK(7)
        if (wid == 0) {
            if (s_full) {
                exchange_topk(val, id, oval, oid, E, K, lane);
                if (lane == 0)
                    for (int q = 0; q < K; q++) s_top[q] = id[q];
            } else {
                exchange_topk(s_cv, s_cid, s_cov, s_coid, nc, K, lane);
                RS_MARK(9)
                if (lane == 0)
                    for (int q = 0; q < K; q++) s_top[q] = s_cid[q];
                RS_MARK(10)
            }
        }
        __syncthreads();
    }

    RS_MARK(3)
    // ---- weights --------------------------------------------------------------
    uint32_t *io = a.idx + (size_t)t * K;
    float *wo = a.w + (size_t)t * K;
    if (warp_done) {
        // written by warp 0 above
    } else if (s_mode == 2) {
        // bit-exact: val holds the reference's probabilities, id the order
        if (tid == 0) {
            float ssum = 0.0f;
            for (int q = 0; q < K; q++) ssum = __fadd_rn(ssum, val[q]);
            for (int q = 0; q < K; q++) {
                io[q] = (uint32_t)id[q];
                wo[q] = a.renorm ? __fdiv_rn(val[q], ssum) : val[q];
            }
        }
    } else {
        const float m = (float)Ls[s_top[0]];
        float sum = 0.f;
        if (a.routing == OFB_ROUTE_FORWARD) {
            for (int e = tid; e < E; e += FR_THREADS) sum += expf((float)Ls[e] - m);
        } else if (tid < K) {
            sum = expf((float)Ls[s_top[tid]] - m);
        }
        sum = block_sum(sum, s_red);
        if (tid < K) s_w[tid] = expf((float)Ls[s_top[tid]] - m) / sum;
        __syncthreads();
        if (tid < K) {
            float ss = 0.f;
            for (int q = 0; q < K; q++) ss += s_w[q];
            io[tid] = (uint32_t)s_top[tid];
            wo[tid] = (a.routing == OFB_ROUTE_FORWARD && a.renorm) ? s_w[tid] / ss : s_w[tid];
        }
    }
    if (tid == 0 && a.stats && !warp_done) atomicAdd(&a.stats[s_mode], 1);
    RS_MARK(4)
    __syncthreads();  // the plan below reuses the shared arrays
    }

    // ---- the block finishing the last token builds the dispatch plan --------
    if (a.T == 1) {
        s_last = 1;
    } else {
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_last = (atomicAdd(a.all_cnt, 1) == a.T - 1);
        }
    }
    __syncthreads();
    if (!s_last) {
        DTRACE_END(rf, 1)
        return;
    }
    if (a.T > 1) __threadfence();
    int *cnt = reinterpret_cast<int *>(smem);
    int *cursor = cnt + 1024;
    __shared__ int wsum[66];
    if (a.plan.n_slots) build_plan(a.plan, cnt, cursor, wsum);
    if (tid == 0) *a.all_cnt = 0;
    DTRACE_END(rf, 1)
}

// ---- large batches: logits and bounds as a tiled fp32 GEMM ---------------------
// For batches above FAST_ROUTE_MAX_T tokens the per-row fp64 dots of
// route_rows_kernel are replaced by a SIMT fp32 GEMM with the same output
// (L~, B) per (token, expert), so route_select_fast certifies the top-k the
// same way:
//  * K runs in 64-element segments; inside a segment the sum is one fp32 FMA
//    chain (each step rounds once), so |c_s - sum_s p| <= gamma_64 * A_s,
//    A_s = sum_s |x w|; segment sums accumulate in fp64: L~ = sum_s c_s.
//  * A_s <= ||x_s|| ||w_s|| (Cauchy-Schwarz) from per-segment norms.
//  * the reference's sequential prefixes P_i (i in segment s) satisfy
//    |P_i| <= |P(64s)| + A_s and |P(64s)| <= |L~ before s| + gamma_64 *
//    (A before s), which bounds S_P = sum |P_i| segment by segment.
//  * B = (1+2^-9) u (A + S_P + n gamma_n A) + (1+2^-9) gamma_64 A + 2^-60,
//    A, S_P accumulated in fp32 rounding up; the norms carry a 2^-16
//    inflation for their own rounding.
constexpr int RG_SEG = 64;

// Norm of every 64-element segment of `rows` rows: one half-warp per segment.
__global__ void segment_norms_kernel(const float *__restrict__ m, int rows, int D, float *__restrict__ nrm) {
    const int nseg = D / RG_SEG;
    const int lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
    const int total = rows * nseg;
    for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; 2 * w < total; w += (gridDim.x * blockDim.x) >> 5) {
        const int i = 2 * w + half;
        float ss = 0.f;
        if (i < total) {
            const int r = i / nseg, sg = i - r * nseg;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(m + (size_t)r * D + sg * RG_SEG) + l16);
            ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (i < total && l16 == 0) nrm[i] = sqrtf(ss) * (1.0f + 0x1.0p-16f);
    }
}

constexpr int RG_LD = RG_SEG + 4;  // smem row stride (floats): 16-byte rows, conflict-free float4 reads
constexpr int RG_THREADS = 128;    // 8 x 16 threads

// Shared memory of a (8 TI) x (16 TJ) output tile: two stages of both
// operand tiles, then the per-thread bound sums (S_P, A) of its TI x TJ outputs.
__host__ __device__ constexpr int rg_smem_ops(int TI, int TJ) { return 2 * (8 * TI + 16 * TJ) * RG_LD * 4; }
__host__ __device__ constexpr int rg_smem(int TI, int TJ) { return rg_smem_ops(TI, TJ) + 2 * TI * TJ * RG_THREADS * 4; }

__device__ __forceinline__ void rg_cp16(float *dst, const float *src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

// Two-stage cp.async pipeline over the 64-element segments; thread (ty, tx)
// owns tokens t0 + ty + 8i (i < TI) and experts e0 + tx + 16j (j < TJ),
// reading float4s along K from [row][k] tiles. TI x TJ = 8 x 4 (64 x 64
// tiles) for large batches; 2 x 2 (16 x 32 tiles) spreads a few hundred
// tokens over enough CTAs to fill the GPU.
template <int TI, int TJ>
__global__ void __launch_bounds__(RG_THREADS) router_bound_gemm(const float *__restrict__ W,
                                                                const float *__restrict__ x,
                                                                const float *__restrict__ nx,
                                                                const float *__restrict__ nw, int T, int D, int E,
                                                                double bound_scale, double ngam, double gam64,
                                                                double2 *__restrict__ cand) {
    constexpr int TT = 8 * TI, TE = 16 * TJ;  // tile tokens, experts
    extern __shared__ __align__(16) float rg_sm[];
    float *xs = rg_sm;                       // [2][TT][RG_LD]
    float *ws = rg_sm + 2 * TT * RG_LD;      // [2][TE][RG_LD]
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    const int nseg = D / RG_SEG;
    const float g64 = (float)gam64;
    auto issue = [&](int sg, int buf) {
#pragma unroll
        for (int q = 0; q < (TT * 16) / RG_THREADS; q++) {
            const int c = tid + RG_THREADS * q, r = c >> 4, kq = c & 15;  // 16 chunks of 16 B per row
            const int tr = min(t0 + r, T - 1);
            rg_cp16(xs + (buf * TT + r) * RG_LD + 4 * kq, x + (size_t)tr * D + sg * RG_SEG + 4 * kq, t0 + r < T);
        }
#pragma unroll
        for (int q = 0; q < (TE * 16) / RG_THREADS; q++) {
            const int c = tid + RG_THREADS * q, r = c >> 4, kq = c & 15;
            const int er = min(e0 + r, E - 1);
            rg_cp16(ws + (buf * TE + r) * RG_LD + 4 * kq, W + (size_t)er * D + sg * RG_SEG + 4 * kq, e0 + r < E);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // bound sums in shared memory, [output slot][thread] (conflict-free)
    float *SPs = rg_sm + rg_smem_ops(TI, TJ) / 4, *Abs = SPs + TI * TJ * RG_THREADS;
    double P[TI][TJ];
#pragma unroll
    for (int i = 0; i < TI; i++)
#pragma unroll
        for (int j = 0; j < TJ; j++) {
            P[i][j] = 0.0;
            SPs[(i * TJ + j) * RG_THREADS + tid] = 0.f;
            Abs[(i * TJ + j) * RG_THREADS + tid] = 0.f;
        }
    issue(0, 0);
    for (int sg = 0; sg < nseg; sg++) {
        const int buf = sg & 1;
        if (sg + 1 < nseg) {
            issue(sg + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        float acc[TI][TJ];
#pragma unroll
        for (int i = 0; i < TI; i++)
#pragma unroll
            for (int j = 0; j < TJ; j++) acc[i][j] = 0.f;
        const float *xb = xs + (buf * TT + ty) * RG_LD, *wb = ws + (buf * TE + tx) * RG_LD;
#pragma unroll 2
        for (int k = 0; k < RG_SEG; k += 4) {
            float4 b[TJ];
#pragma unroll
            for (int j = 0; j < TJ; j++) b[j] = *reinterpret_cast<const float4 *>(wb + 16 * j * RG_LD + k);
            // the segment's chain runs in k order: one FMA per step and output
#pragma unroll
            for (int i = 0; i < TI; i++) {
                const float4 av = *reinterpret_cast<const float4 *>(xb + 8 * i * RG_LD + k);
#pragma unroll
                for (int j = 0; j < TJ; j++) {
                    acc[i][j] = fmaf(av.x, b[j].x, acc[i][j]);
                    acc[i][j] = fmaf(av.y, b[j].y, acc[i][j]);
                    acc[i][j] = fmaf(av.z, b[j].z, acc[i][j]);
                    acc[i][j] = fmaf(av.w, b[j].w, acc[i][j]);
                }
            }
        }
        // fold the segment: prefix bound with the sums before it, then the sum
        float wn[TJ];
#pragma unroll
        for (int j = 0; j < TJ; j++) wn[j] = nw[(size_t)min(e0 + tx + 16 * j, E - 1) * nseg + sg];
#pragma unroll
        for (int i = 0; i < TI; i++) {
            const float xn = nx[(size_t)min(t0 + ty + 8 * i, T - 1) * nseg + sg];
#pragma unroll
            for (int j = 0; j < TJ; j++) {
                float *sp = SPs + (i * TJ + j) * RG_THREADS + tid, *ab = Abs + (i * TJ + j) * RG_THREADS + tid;
                const float as = __fmul_ru(xn, wn[j]), a0 = *ab;
                const float pb = __fmaf_ru(g64, a0, __double2float_ru(fabs(P[i][j])));
                *sp = __fmaf_ru(64.f, __fadd_ru(pb, as), *sp);
                *ab = __fadd_ru(a0, as);
                P[i][j] += (double)acc[i][j];
            }
        }
        __syncthreads();  // this buffer is refilled two segments on
    }
#pragma unroll
    for (int i = 0; i < TI; i++) {
        const int t = t0 + ty + 8 * i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < TJ; j++) {
            const int e = e0 + tx + 16 * j;
            if (e >= E) continue;
            const double A = Abs[(i * TJ + j) * RG_THREADS + tid];
            const double B = bound_scale * (A + (double)SPs[(i * TJ + j) * RG_THREADS + tid] + ngam * A) +
                             (1.0 + 0x1.0p-9) * gam64 * A + 0x1.0p-60;
            cand[(size_t)t * E + e] = make_double2(P[i][j], B);
        }
    }
}

// ---- batches below 1024 tokens: the same (L~, B), split over segments -------
// router_bound_gemm walks the 32 segments of a tile in order, so a few
// hundred tokens give ~128 CTAs each with a long serial loop. The segment
// sums c_s do not depend on each other: router_seg_gemm computes them with
// one CTA per (64-token tile, 64-expert tile, segment) - the same fp32
// FMA chain per segment, in the same k order - into segsum[s][t][e], and
// router_seg_scan then runs router_bound_gemm's per-segment recurrence (the
// fp64 sum and the bound terms, the same operations in the same order) for
// one (token, expert) per thread. Results are identical to router_bound_gemm.
constexpr int RS_SEGS = 1;  // segments per CTA (up to two cp.async stages)
__global__ void __launch_bounds__(RG_THREADS) router_seg_gemm(const float *__restrict__ W, const float *__restrict__ x,
                                                              int T, int D, int E, float *__restrict__ segsum) {
    constexpr int TI = 8, TJ = 4, TT = 8 * TI, TE = 16 * TJ;
    extern __shared__ __align__(16) float rg_sm[];
    float *xs = rg_sm;                   // [2][TT][RG_LD]
    float *ws = rg_sm + 2 * TT * RG_LD;  // [2][TE][RG_LD]
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE, sg0 = blockIdx.z * RS_SEGS;
    const int nseg = D / RG_SEG, ns = min(RS_SEGS, nseg - sg0);
    auto issue = [&](int sg, int buf) {
#pragma unroll
        for (int q = 0; q < (TT * 16) / RG_THREADS; q++) {
            const int c = tid + RG_THREADS * q, r = c >> 4, kq = c & 15;
            const int tr = min(t0 + r, T - 1);
            rg_cp16(xs + (buf * TT + r) * RG_LD + 4 * kq, x + (size_t)tr * D + sg * RG_SEG + 4 * kq, t0 + r < T);
        }
#pragma unroll
        for (int q = 0; q < (TE * 16) / RG_THREADS; q++) {
            const int c = tid + RG_THREADS * q, r = c >> 4, kq = c & 15;
            const int er = min(e0 + r, E - 1);
            rg_cp16(ws + (buf * TE + r) * RG_LD + 4 * kq, W + (size_t)er * D + sg * RG_SEG + 4 * kq, e0 + r < E);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int q = 0; q < ns; q++) issue(sg0 + q, q);
    for (int q = 0; q < ns; q++) {
        if (q + 1 < ns) asm volatile("cp.async.wait_group 1;" ::: "memory");
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        float acc[TI][TJ];
#pragma unroll
        for (int i = 0; i < TI; i++)
#pragma unroll
            for (int j = 0; j < TJ; j++) acc[i][j] = 0.f;
        const float *xb = xs + (q * TT + ty) * RG_LD, *wb = ws + (q * TE + tx) * RG_LD;
#pragma unroll 2
        for (int k = 0; k < RG_SEG; k += 4) {
            float4 b[TJ];
#pragma unroll
            for (int j = 0; j < TJ; j++) b[j] = *reinterpret_cast<const float4 *>(wb + 16 * j * RG_LD + k);
#pragma unroll
            for (int i = 0; i < TI; i++) {
                const float4 av = *reinterpret_cast<const float4 *>(xb + 8 * i * RG_LD + k);
#pragma unroll
                for (int j = 0; j < TJ; j++) {
                    acc[i][j] = fmaf(av.x, b[j].x, acc[i][j]);
                    acc[i][j] = fmaf(av.y, b[j].y, acc[i][j]);
                    acc[i][j] = fmaf(av.z, b[j].z, acc[i][j]);
                    acc[i][j] = fmaf(av.w, b[j].w, acc[i][j]);
                }
            }
        }
        float *out = segsum + (size_t)(sg0 + q) * T * E;
#pragma unroll
        for (int i = 0; i < TI; i++) {
            const int t = t0 + ty + 8 * i;
            if (t >= T) continue;
#pragma unroll
            for (int j = 0; j < TJ; j++) {
                const int e = e0 + tx + 16 * j;
                if (e < E) out[(size_t)t * E + e] = acc[i][j];
            }
        }
    }
}

__global__ void __launch_bounds__(256) router_seg_scan(const float *__restrict__ segsum, const float *__restrict__ nx,
                                                       const float *__restrict__ nw, int T, int D, int E,
                                                       double bound_scale, double ngam, double gam64,
                                                       double2 *__restrict__ cand) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * E) return;
    const int t = i / E, e = i - t * E, nseg = D / RG_SEG;
    const float g64 = (float)gam64;
    double P = 0.0;
    float SP = 0.f, Ab = 0.f;
    // this expert's segment norms, 16 bytes at a time (a warp's threads are
    // nseg floats apart, so one float per load would touch a sector each)
    const float4 *nw4 = reinterpret_cast<const float4 *>(nw + (size_t)e * nseg);
    float4 wq = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sg = 0; sg < nseg; sg++) {
        if ((sg & 3) == 0) wq = __ldg(nw4 + (sg >> 2));
        const float wn = (sg & 3) == 0 ? wq.x : (sg & 3) == 1 ? wq.y : (sg & 3) == 2 ? wq.z : wq.w;
        const float c = __ldg(segsum + (size_t)sg * T * E + i);
        const float as = __fmul_ru(__ldg(nx + (size_t)t * nseg + sg), wn), a0 = Ab;
        const float pb = __fmaf_ru(g64, a0, __double2float_ru(fabs(P)));
        SP = __fmaf_ru(64.f, __fadd_ru(pb, as), SP);
        Ab = __fadd_ru(a0, as);
        P += (double)c;
    }
    const double A = Ab;
    const double B = bound_scale * (A + (double)SP + ngam * A) + (1.0 + 0x1.0p-9) * gam64 * A + 0x1.0p-60;
    cand[i] = make_double2(P, B);
}

template <int TI, int TJ>
static void launch_rg(const float *W, const float *x, const float *nx, const float *nw, int T, int D, int E,
                      double bound_scale, double ngam, double gam64, double2 *cand, cudaStream_t s) {
    cudaFuncSetAttribute(router_bound_gemm<TI, TJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, rg_smem(TI, TJ));
    router_bound_gemm<TI, TJ><<<dim3((T + 8 * TI - 1) / (8 * TI), (E + 16 * TJ - 1) / (16 * TJ)), RG_THREADS,
                                rg_smem(TI, TJ), s>>>(W, x, nx, nw, T, D, E, bound_scale, ngam, gam64, cand);
}

size_t route_fast_smem(int E, int D) {
    size_t sel = xl_offset(E, D) + XL_SMEM;
    size_t plan = 2 * 1024 * sizeof(int);
    return sel > plan ? sel : plan;
}

int launch_route_fast(const float *W, const float *x, const float *gate_v, int T, int D, int E, int K,
                      int routing, int renorm, double2 *cand, int *all_cnt, int *stats,
                      uint32_t *idx, float *w, float *gsc, unsigned char *xq, const PlanArgs *plan,
                      cudaStream_t s) {
    FastRouteArgs a;
    a.W = W; a.x = x; a.gate_v = gate_v;
    a.T = T; a.D = D; a.E = E; a.K = K; a.routing = routing; a.renorm = renorm;
    const double u = 0x1.0p-24, n = (double)D;
    a.bound_scale = (1.0 + 0x1.0p-9) * u;
    a.ngam = n * (n * u / (1.0 - n * u));
    a.cand = cand; a.all_cnt = all_cnt; a.stats = stats;
    a.idx = idx; a.w = w; a.gsc = gsc; a.xq = xq;
    if (plan) a.plan = *plan;
    else memset(&a.plan, 0, sizeof(a.plan));
    a.flagged = nullptr;
    a.n_flagged = nullptr;
    const size_t smem = route_fast_smem(E, D);
    static size_t attr[64];
    cudaError_t ea = ensure_dyn_smem(route_select_fast, (size_t)FR_SMEM_MAX, attr);
    if (ea != cudaSuccess) return cuda_status(ea, "route_select_fast smem attribute");
    if (smem > FR_SMEM_MAX) { set_error("route_fast: E/D too large for shared memory"); return OFB_EUNSUPPORTED; }
    // rows: E router rows, the gate vector, then (when x is quantised) one
    // warp per 32-element sub-block of x
    const int rr_rows = E + 1 + (xq ? D / 32 : 0);
    // rows per block: 8 while the staged rows fit comfortably, fewer for wide rows
    int rw = RR_WARPS;
    while (rw > 1 && rr_smem(D, rw) > 120 * 1024) rw >>= 1;
    const size_t rsm = rr_smem(D, rw);
    if (rsm > 227 * 1024) { set_error("route_fast: d_model %d too large for the row kernel", D); return OFB_EUNSUPPORTED; }
    static size_t rr_attr[64];
    cudaError_t e = ensure_dyn_smem(route_rows_kernel, rsm, rr_attr);
    if (e != cudaSuccess) return cuda_status(e, "route_rows smem attribute");
    e = launch_pdl(route_rows_kernel, dim3((rr_rows + rw - 1) / rw, T), dim3(rw * 32), rsm, s, a);
    if (e == cudaSuccess) e = launch_pdl(route_select_fast, dim3(T), dim3(FR_THREADS), smem, s, a);
    if (e != cudaSuccess) return cuda_status(e, "route_fast launch");
    return OFB_OK;
}

int launch_route_fast_large(const float *W, const float *x, const float *gate_v, float *gsc, int T, int D, int E,
                            int K, int routing, int renorm, double2 *cand, float *norms, float *segsum, int *flagged, int *n_flagged, int *stats,
                            uint32_t *idx, float *w, cudaStream_t s) {
    if (D % RG_SEG) { set_error("route_fast_large: d_model must be a multiple of %d", RG_SEG); return OFB_EUNSUPPORTED; }
    FastRouteArgs a;
    a.W = W; a.x = x; a.gate_v = gate_v;  // with gsc: the shared-expert gates, by the certify warps
    a.T = T; a.D = D; a.E = E; a.K = K; a.routing = routing; a.renorm = renorm;
    const double u = 0x1.0p-24, n = (double)D;
    a.bound_scale = (1.0 + 0x1.0p-9) * u;
    a.ngam = n * (n * u / (1.0 - n * u));
    const double gam64 = 64.0 * u / (1.0 - 64.0 * u);
    a.cand = cand; a.all_cnt = nullptr; a.stats = stats;
    a.idx = idx; a.w = w; a.gsc = gate_v ? gsc : nullptr; a.xq = nullptr;
    memset(&a.plan, 0, sizeof(a.plan));
    a.flagged = flagged;
    a.n_flagged = n_flagged;
    const size_t smem = route_fast_smem(E, D);
    if (smem > FR_SMEM_MAX) { set_error("route_fast: E/D too large for shared memory"); return OFB_EUNSUPPORTED; }
    cudaFuncSetAttribute(route_select_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, FR_SMEM_MAX);
    float *nx = norms, *nw = norms + (size_t)T * (D / RG_SEG);
    const int nseg = D / RG_SEG;
    segment_norms_kernel<<<grid_for((uint64_t)T * nseg / 2, 8, 148 * 16), 256, 0, s>>>(x, T, D, nx);
    segment_norms_kernel<<<grid_for((uint64_t)E * nseg / 2, 8, 148 * 16), 256, 0, s>>>(W, E, D, nw);
    if (T >= ROUTE_SPLIT_MAX_T || !segsum) {
        if (T >= 1024) launch_rg<8, 4>(W, x, nx, nw, T, D, E, a.bound_scale, a.ngam, gam64, cand, s);
        else launch_rg<2, 2>(W, x, nx, nw, T, D, E, a.bound_scale, a.ngam, gam64, cand, s);
    } else {
        const int ops = rg_smem_ops(8, 4);
        cudaFuncSetAttribute(router_seg_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, ops);
        router_seg_gemm<<<dim3((T + 63) / 64, (E + 63) / 64, (nseg + RS_SEGS - 1) / RS_SEGS), RG_THREADS, ops, s>>>(
            W, x, T, D, E, segsum);
        router_seg_scan<<<(T * E + 255) / 256, 256, 0, s>>>(segsum, nx, nw, T, D, E, a.bound_scale, a.ngam, gam64,
                                                           cand);
    }
    if (E > 32 * FW_PER_LANE) { set_error("route_fast_large: at most %d experts", 32 * FW_PER_LANE); return OFB_EUNSUPPORTED; }
    cudaError_t e = cudaMemsetAsync(n_flagged, 0, sizeof(int), s);
    if (e != cudaSuccess) return cuda_status(e, "route_fast_large memset");
    route_certify_warps<<<(T + 7) / 8, 256, 0, s>>>(a, flagged, n_flagged);
    // flagged tokens, one warp each, all at once (blocks past the flagged
    // count exit at once)
    const size_t fb_smem = FB_WARPS * fb_warp_smem(E, D);
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x)) & 15) {
        set_error("route_fast_large: router and activations must be 16-byte aligned");
        return OFB_EINVAL;
    }
    if (fb_smem > 227 * 1024 || D % FB_CK) {
        set_error("route_fast_large: d_model %d / %d experts do not fit the fallback", D, E);
        return OFB_EUNSUPPORTED;
    }
    cudaFuncSetAttribute(route_fallback_warps, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fb_smem);
    route_fallback_warps<<<(T + FB_WARPS - 1) / FB_WARPS, FB_WARPS * 32, fb_smem, s>>>(a);
    OFB_CHECK_LAUNCH("route_fast_large");
    return OFB_OK;
}

}  // namespace ofb
