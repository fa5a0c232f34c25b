// route_fast.cu — certified routing for decode-sized batches, with the
// shared-expert gates and the dispatch plan built in the same launch.
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
//  2. The last block to finish a token (atomic ticket) ranks the experts by L~
//     and CERTIFIES the reference's top-k: every adjacent gap in the top-k
//     and the gap to every other expert must exceed the two bounds plus a
//     margin M = 2^-14, large enough that expf(l - max) and the divided
//     probabilities stay strictly ordered after fp32 rounding. Then the
//     reference's exchange sort (model.c:1042-1049), which only ever swaps on
//     strict '>', yields exactly this order: the indices are bit-exact.
//  3. Otherwise (rare: two logits closer than ~1e-4) the block recomputes the
//     uncertain candidates with the reference's exact sequential chain and the
//     host library's expf (exact_expf.h), and emulates the exchange sort on
//     them; if two candidate probabilities could round together, it
//     recomputes every expert exactly (bit-exact softmax sum) before sorting.
// Routing weights come from fp32 softmax of L~ (or the exact logits where
// computed): within ~1e-6 relative of the reference's (bit-exact in the
// full-recompute case). The last token's block builds the dispatch plan.
// Interleaved-layout routers and large batches use the exact kernels of
// route.cu.
#include "common.cuh"
#include "exact_expf.h"
#include "moe.cuh"
#include "route.cuh"
#include "exchange.cuh"
#include "plan.cuh"

namespace ofb {

constexpr int FR_WARPS = 8;
constexpr double FR_MARGIN = 0x1.0p-14;

struct FastRouteArgs {
    const float *W, *x, *gate_v;
    int T, D, E, K, routing, renorm;
    double2 *cand;  // [T][E+1]: (L~, B)
    int *tok_cnt;   // [T], zero between calls
    int *all_cnt;   // [1], zero between calls
    int *stats;     // [3]: certified, candidate recompute, full recompute
    uint32_t *idx;
    float *w, *gsc;
    PlanArgs plan;
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Reference-order logit: sequential fp32, product then add, d = 0..D-1.
__device__ float exact_logit(const float *wrow, const float *xs, int D) {
    float s = 0.0f;
    const float4 *w4 = reinterpret_cast<const float4 *>(wrow);
#pragma unroll 4
    for (int i = 0; i < D / 4; i++) {
        float4 w = __ldg(w4 + i);
        s = __fadd_rn(s, __fmul_rn(xs[4 * i + 0], w.x));
        s = __fadd_rn(s, __fmul_rn(xs[4 * i + 1], w.y));
        s = __fadd_rn(s, __fmul_rn(xs[4 * i + 2], w.z));
        s = __fadd_rn(s, __fmul_rn(xs[4 * i + 3], w.w));
    }
    return s;
}

__device__ __forceinline__ bool close_ulps(float a, float b, int ulps) {
    int ia = __float_as_int(a), ib = __float_as_int(b);  // non-negative floats
    return abs(ia - ib) <= ulps;
}

__global__ void __launch_bounds__(FR_WARPS * 32) route_fast_kernel(FastRouteArgs a) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int t = blockIdx.y;
    const int E = a.E, D = a.D, K = a.K;
    const int r = blockIdx.x * FR_WARPS + wid;  // router row; r == E is the gate vector
    const float *xt = a.x + (size_t)t * D;

    // ---- 1. approximate logit + bound, one warp per row -------------------
    const bool has_row = (r < E) || (r == E && a.gate_v);
    if (has_row) {
        const float *wr = (r < E) ? a.W + (size_t)r * D : a.gate_v;
        const int seg = D / 32;  // multiple of 8
        const float4 *w4 = reinterpret_cast<const float4 *>(wr + lane * seg);
        const float4 *x4 = reinterpret_cast<const float4 *>(xt + lane * seg);
        double P = 0.0, SP = 0.0, A = 0.0;
        for (int i = 0; i < seg / 4; i++) {
            const float4 wv = __ldg(w4 + i), xv = __ldg(x4 + i);
            const double p0 = (double)xv.x * wv.x, p1 = (double)xv.y * wv.y;
            const double p2 = (double)xv.z * wv.z, p3 = (double)xv.w * wv.w;
            P += p0; SP += fabs(P);
            P += p1; SP += fabs(P);
            P += p2; SP += fabs(P);
            P += p3; SP += fabs(P);
            A += fabs(p0) + fabs(p1) + fabs(p2) + fabs(p3);
        }
        // exclusive scan of segment sums -> |prefix| bound of this segment
        double inc = P;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double up = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += up;
        }
        const double base = inc - P;
        const double sp_bound = (double)seg * fabs(base) + SP;
        const double L = warp_sum_d(P);
        const double SPt = warp_sum_d(sp_bound);
        const double At = warp_sum_d(A);
        if (lane == 0) {
            if (r < E) {
                const double u = 0x1.0p-24, n = (double)D;
                const double gam = n * u / (1.0 - n * u);
                const double B = (1.0 + 0x1.0p-9) * u * (At + SPt + n * gam * At) + 0x1.0p-60;
                a.cand[(size_t)t * (E + 1) + r] = make_double2(L, B);
            } else {
                a.gsc[t] = 1.0f / (1.0f + expf(-(float)L));
            }
        }
    }

    // ---- last block of this token does the selection ------------------------
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = (atomicAdd(&a.tok_cnt[t], 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    extern __shared__ __align__(16) unsigned char smem[];
    double *Ls = reinterpret_cast<double *>(smem);     // [E]
    double *Bs = Ls + E;                                // [E]
    float *val = reinterpret_cast<float *>(Bs + E);     // [E]
    int *id = reinterpret_cast<int *>(val + E);         // [E]
    float *oval = reinterpret_cast<float *>(id + E);    // [E]
    int *oid = reinterpret_cast<int *>(oval + E);       // [E]
    float *xs = reinterpret_cast<float *>(oid + E);     // [D]
    int *taken = reinterpret_cast<int *>(xs + D);       // [E]
    __shared__ int s_top[17];
    __shared__ int s_mode;  // 0 certified, 1 candidate recompute, 2 full recompute
    __shared__ float s_ex[16];

    const double2 *cd = a.cand + (size_t)t * (E + 1);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        double2 v = __ldcg(cd + e);
        Ls[e] = v.x;
        Bs[e] = v.y;
        taken[e] = 0;
    }
    __syncthreads();

    if (wid == 0) {
        // top-k by L~ (ties: lower index first)
        const int kk = K < E ? K + 1 : K;
        for (int it = 0; it < kk; it++) {
            double bv = -INFINITY;
            int be = 0x7fffffff;
            for (int e = lane; e < E; e += 32)
                if (!taken[e] && (Ls[e] > bv || (Ls[e] == bv && e < be))) { bv = Ls[e]; be = e; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                double ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oe = __shfl_xor_sync(0xffffffffu, be, o);
                if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
            }
            if (it < K) {
                if (lane == 0) { s_top[it] = be; taken[be] = 1; }
            }
            __syncwarp();
        }
        // largest upper bound outside the top-k
        double hi_rest = -INFINITY;
        for (int e = lane; e < E; e += 32)
            if (!taken[e]) hi_rest = fmax(hi_rest, Ls[e] + Bs[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) hi_rest = fmax(hi_rest, __shfl_xor_sync(0xffffffffu, hi_rest, o));
        if (lane == 0) {
            bool ok = true;
            for (int q = 0; q + 1 < K; q++) {
                const int e0 = s_top[q], e1 = s_top[q + 1];
                ok = ok && (Ls[e0] - Bs[e0] > Ls[e1] + Bs[e1] + FR_MARGIN);
            }
            const int el = s_top[K - 1];
            ok = ok && (Ls[el] - Bs[el] > hi_rest + FR_MARGIN);
            ok = ok && (Ls[el] - Ls[s_top[0]] > -80.0);
            s_mode = ok ? 0 : 1;
        }
        __syncwarp();
    }
    __syncthreads();

    if (s_mode != 0) {
        // ---- candidate recompute with the reference's exact chain --------
        for (int d = threadIdx.x; d < D; d += blockDim.x) xs[d] = xt[d];
        double lo_min = INFINITY;
        for (int q = 0; q < K; q++) lo_min = fmin(lo_min, Ls[s_top[q]] - Bs[s_top[q]]);
        __syncthreads();
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            const bool cand = (Ls[e] + Bs[e] >= lo_min - FR_MARGIN);
            val[e] = cand ? exact_logit(a.W + (size_t)e * D, xs, D) : -INFINITY;
            id[e] = e;
            taken[e] = cand;
        }
        __syncthreads();
        if (a.routing == OFB_ROUTE_FORWARD) {
            // probabilities are ordered like expf(l - max) unless two of them
            // are within a few ulps (then the division could tie them)
            __shared__ float s_max;
            if (threadIdx.x == 0) {
                float m = -INFINITY;
                for (int e = 0; e < E; e++)
                    if (taken[e]) m = fmaxf(m, val[e]);
                s_max = m;
            }
            __syncthreads();
            for (int e = threadIdx.x; e < E; e += blockDim.x)
                oval[e] = taken[e] ? ofb_exact_expf(__fsub_rn(val[e], s_max)) : -INFINITY;
            __syncthreads();
            __shared__ int s_unsafe;
            if (threadIdx.x == 0) s_unsafe = 0;
            __syncthreads();
            for (int e = threadIdx.x; e < E; e += blockDim.x) {
                if (!taken[e]) continue;
                for (int f = 0; f < E; f++)
                    if (f != e && taken[f] && close_ulps(oval[e], oval[f], 4)) s_unsafe = 1;
            }
            __syncthreads();
            if (s_unsafe) {
                // ---- full recompute: every logit exact, softmax as the reference
                for (int e = threadIdx.x; e < E; e += blockDim.x)
                    val[e] = taken[e] ? val[e] : exact_logit(a.W + (size_t)e * D, xs, D);
                __syncthreads();
                if (threadIdx.x == 0) {
                    float m = val[0];
                    for (int e = 1; e < E; e++) if (val[e] > m) m = val[e];
                    s_max = m;
                }
                __syncthreads();
                for (int e = threadIdx.x; e < E; e += blockDim.x)
                    val[e] = ofb_exact_expf(__fsub_rn(val[e], s_max));
                __syncthreads();
                __shared__ float s_sum;
                if (threadIdx.x == 0) {
                    float s = 0.0f;
                    for (int e = 0; e < E; e++) s = __fadd_rn(s, val[e]);
                    s_sum = s;
                    s_mode = 2;
                }
                __syncthreads();
                for (int e = threadIdx.x; e < E; e += blockDim.x) val[e] = __fdiv_rn(val[e], s_sum);
            } else {
                for (int e = threadIdx.x; e < E; e += blockDim.x) val[e] = oval[e];
            }
            __syncthreads();
        }
        if (wid == 0) {
            for (int i = 0; i < K; i++) exchange_pass(val, id, oval, oid, E, i, lane);
            if (lane == 0)
                for (int q = 0; q < K; q++) s_top[q] = id[q];
        }
        __syncthreads();
    }

    // ---- weights --------------------------------------------------------------
    if (wid == 0) {
        uint32_t *io = a.idx + (size_t)t * K;
        float *wo = a.w + (size_t)t * K;
        if (s_mode == 2) {
            // bit-exact: val holds the reference's probabilities, id the order
            if (lane == 0) {
                float ssum = 0.0f;
                for (int q = 0; q < K; q++) ssum = __fadd_rn(ssum, val[q]);
                for (int q = 0; q < K; q++) {
                    io[q] = (uint32_t)id[q];
                    wo[q] = a.renorm ? __fdiv_rn(val[q], ssum) : val[q];
                }
            }
        } else {
            const float m = (float)Ls[s_top[0]];
            if (a.routing == OFB_ROUTE_GET_ROUTING) {
                if (lane < K) s_ex[lane] = expf((float)Ls[s_top[lane]] - m);
                __syncwarp();
                if (lane == 0) {
                    float s = 0.0f;
                    for (int q = 0; q < K; q++) s += s_ex[q];
                    for (int q = 0; q < K; q++) { io[q] = (uint32_t)s_top[q]; wo[q] = s_ex[q] / s; }
                }
            } else {
                float s = 0.0f;
                for (int e = lane; e < E; e += 32) s += expf((float)Ls[e] - m);
                s = warp_sum(s);
                if (lane < K) s_ex[lane] = expf((float)Ls[s_top[lane]] - m) / s;
                __syncwarp();
                if (lane == 0) {
                    float ss = 0.0f;
                    for (int q = 0; q < K; q++) ss += s_ex[q];
                    for (int q = 0; q < K; q++) {
                        io[q] = (uint32_t)s_top[q];
                        wo[q] = a.renorm ? s_ex[q] / ss : s_ex[q];
                    }
                }
            }
        }
        if (lane == 0) {
            if (a.stats) atomicAdd(&a.stats[s_mode], 1);
            a.tok_cnt[t] = 0;
        }
    }

    // ---- the block finishing the last token builds the dispatch plan --------
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = (atomicAdd(a.all_cnt, 1) == a.T - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    int *cnt = reinterpret_cast<int *>(smem);
    int *cursor = cnt + 1024;
    __shared__ int wsum[66];
    if (a.plan.n_slots) build_plan(a.plan, cnt, cursor, wsum);
    if (threadIdx.x == 0) *a.all_cnt = 0;
}

size_t route_fast_smem(int E, int D) {
    size_t sel = (size_t)E * (8 + 8 + 4 + 4 + 4 + 4 + 4) + (size_t)D * 4;
    size_t plan = 2 * 1024 * sizeof(int);
    return sel > plan ? sel : plan;
}

int launch_route_fast(const float *W, const float *x, const float *gate_v, int T, int D, int E, int K,
                      int routing, int renorm, double2 *cand, int *tok_cnt, int *all_cnt, int *stats,
                      uint32_t *idx, float *w, float *gsc, const PlanArgs *plan, cudaStream_t s) {
    FastRouteArgs a;
    a.W = W; a.x = x; a.gate_v = gate_v;
    a.T = T; a.D = D; a.E = E; a.K = K; a.routing = routing; a.renorm = renorm;
    a.cand = cand; a.tok_cnt = tok_cnt; a.all_cnt = all_cnt; a.stats = stats;
    a.idx = idx; a.w = w; a.gsc = gsc;
    if (plan) a.plan = *plan;
    else memset(&a.plan, 0, sizeof(a.plan));
    const size_t smem = route_fast_smem(E, D);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(route_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        attr_set = true;
    }
    if (smem > 64 * 1024) { set_error("route_fast: E/D too large for shared memory"); return OFB_EUNSUPPORTED; }
    dim3 grid((E + 1 + FR_WARPS - 1) / FR_WARPS, T);
    route_fast_kernel<<<grid, FR_WARPS * 32, smem, s>>>(a);
    OFB_CHECK_LAUNCH("route_fast");
    return OFB_OK;
}

}  // namespace ofb
