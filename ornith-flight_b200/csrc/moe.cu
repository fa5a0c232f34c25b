// moe.cu — the MoE feed-forward layer: dispatch plan, expert SwiGLU and the
// weighted combine (the block engine/src/model.c:992-1143, batched).
//
// Pipeline for n tokens (all stream-ordered, no host synchronisation):
//   1. routing: certified fast kernels for decode batches (route_fast.cu),
//      the exact kernels otherwise (route.cu); idx[T][K], w[T][K].
//   2. dispatch plan (plan.cuh): device histogram of the kept assignments per
//      expert, scan, and a CSR "slot" list: slot u = one used expert
//      (ascending id) with its assignment ids; the shared expert is the last
//      slot with every token. Assignment id a < T*K is (token a/K, rank a%K);
//      a >= T*K is the shared expert of token a-T*K.
//   3. experts: decode batches (T <= 32) use the dp4a GEMV kernels of
//      decode.cu; larger batches the tcgen05 grouped GEMMs of prefill.cu.
// The interleaved (reference-slice) layout uses the element-wise kernels
// below; it touches every block of a tensor by construction and is the
// correctness path for that layout.
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "moe.cuh"
#include "route.cuh"
#include "plan.cuh"

namespace ofb {

__device__ __forceinline__ float silu_ref(float g) {
    // engine/src/model.c:340-344
    if (g < -50.0f) return 0.0f;
    if (g > 50.0f) return g;
    return g / (1.0f + expf(-g));
}

__device__ __forceinline__ int asg_token(int a, int TK, int K) { return a < TK ? a / K : a - TK; }

// ---- dispatch plan over many CTAs ------------------------------------------------
// The CSR plan of build_plan (kept routed assignments grouped by expert in
// ascending expert order, then the shared slot) for large batches, in three
// launches: CTA b counts the kept assignments [b*PLAN_CH, (b+1)*PLAN_CH) per
// expert (hist[b][e]); one block turns the counts into each CTA's first
// position per expert, the slot list and (for the tensor-core path) the tile
// list; CTA b then places its assignments. Within one expert the
// assignments of a CTA land in any order (the expert kernels treat every row
// on its own).
__global__ void __launch_bounds__(256) plan_hist_kernel(PlanArgs p, int *__restrict__ hist) {
    __shared__ int cnt[1024];
    const int tid = threadIdx.x, TK = p.T * p.K, i0 = blockIdx.x * PLAN_CH, i1 = min(TK, i0 + PLAN_CH);
    for (int e = tid; e < p.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = i0 + tid; i < i1; i += blockDim.x)
        if (!(__ldcg(p.w + i) < 1e-6f)) atomicAdd(&cnt[__ldcg(p.idx + i)], 1);  // model.c:1066 skip rule
    __syncthreads();
    for (int e = tid; e < p.E; e += blockDim.x) hist[(size_t)blockIdx.x * p.E + e] = cnt[e];
}

// One block of 1024 threads, thread e owning expert e (E <= 1024). hist[b][e]
// becomes CTA b's offset inside expert e's run, hist[nb][e] the run's start,
// hist[nb][E] the number of kept routed assignments.
__global__ void __launch_bounds__(1024) plan_scan_kernel(PlanArgs p, int *__restrict__ hist, int nb,
                                                         int *__restrict__ tiles, int max_tiles) {
    __shared__ int ws[32][3], tot[3];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, E = p.E;
    int c = 0;
    if (tid < E)
        for (int b0 = 0; b0 < nb; b0 += 16) {
            // 16 counts loaded before any store (independent loads in flight)
            int v[16];
#pragma unroll
            for (int q = 0; q < 16; q++) v[q] = b0 + q < nb ? hist[(size_t)(b0 + q) * E + tid] : 0;
#pragma unroll
            for (int q = 0; q < 16; q++) {
                if (b0 + q < nb) hist[(size_t)(b0 + q) * E + tid] = c;
                c += v[q];
            }
        }
    // exclusive scans over experts of (has slot, count, tiles)
    const int nt = (c + PF_NMAX - 1) / PF_NMAX;
    int v[3] = {c > 0, c, nt}, inc[3] = {v[0], v[1], v[2]};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
#pragma unroll
        for (int q = 0; q < 3; q++) {
            const int u = __shfl_up_sync(0xffffffffu, inc[q], o);
            if (lane >= o) inc[q] += u;
        }
    if (lane == 31)
        for (int q = 0; q < 3; q++) ws[wid][q] = inc[q];
    __syncthreads();
    if (wid == 0) {
        int a[3], ai[3];
        for (int q = 0; q < 3; q++) ai[q] = a[q] = ws[lane][q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
#pragma unroll
            for (int q = 0; q < 3; q++) {
                const int u = __shfl_up_sync(0xffffffffu, ai[q], o);
                if (lane >= o) ai[q] += u;
            }
        for (int q = 0; q < 3; q++) {
            ws[lane][q] = ai[q] - a[q];
            if (lane == 31) tot[q] = ai[q];
        }
    }
    __syncthreads();
    const int F = inc[0] - v[0] + ws[wid][0], C = inc[1] - v[1] + ws[wid][1], Tb = inc[2] - v[2] + ws[wid][2];
    int *n_tiles = tiles, *tile_slot = tiles + 1, *tile_start = tile_slot + max_tiles, *tile_n = tile_start + max_tiles;
    if (tid < E) {
        hist[(size_t)nb * E + tid] = C;
        if (c > 0) {
            p.slot_expert[F] = tid;
            p.slot_start[F] = C;
            if (tiles)
                for (int k = 0; k < nt; k++) {
                    tile_slot[Tb + k] = F;
                    tile_start[Tb + k] = C + k * PF_NMAX;
                    tile_n[Tb + k] = min(PF_NMAX, c - k * PF_NMAX);
                }
        }
    }
    if (tid == 0) {
        const int ns = tot[0], total = tot[1];
        int u = ns, ntl = tot[2];
        hist[(size_t)nb * E + E] = total;
        if (p.has_shared) {
            p.slot_expert[u] = E;
            p.slot_start[u] = total;
            if (tiles)
                for (int k = 0; k * PF_NMAX < p.T; k++, ntl++) {
                    tile_slot[ntl] = u;
                    tile_start[ntl] = total + k * PF_NMAX;
                    tile_n[ntl] = min(PF_NMAX, p.T - k * PF_NMAX);
                }
            u++;
            p.slot_start[u] = total + p.T;
        } else {
            p.slot_start[u] = total;
        }
        *p.n_slots = u;
        if (tiles) *n_tiles = ntl;
    }
}

__global__ void __launch_bounds__(256) plan_scatter_kernel(PlanArgs p, const int *__restrict__ hist, int nb) {
    __shared__ int cur[1024];
    const int tid = threadIdx.x, E = p.E, TK = p.T * p.K, i0 = blockIdx.x * PLAN_CH, i1 = min(TK, i0 + PLAN_CH);
    for (int e = tid; e < E; e += blockDim.x) cur[e] = hist[(size_t)blockIdx.x * E + e] + hist[(size_t)nb * E + e];
    __syncthreads();
    for (int i = i0 + tid; i < i1; i += blockDim.x)
        if (!(__ldcg(p.w + i) < 1e-6f)) p.assign[atomicAdd(&cur[__ldcg(p.idx + i)], 1)] = i;
    if (p.has_shared) {
        const int total = hist[(size_t)nb * E + E];
        for (int t = blockIdx.x * blockDim.x + tid; t < p.T; t += gridDim.x * blockDim.x) p.assign[total + t] = TK + t;
    }
}

int launch_plan(const PlanArgs &p, int *hist, int *tiles, int max_tiles, cudaStream_t s) {
    if (p.E > 1024) { set_error("plan: at most 1024 experts"); return OFB_EUNSUPPORTED; }
    const int nb = (p.T * p.K + PLAN_CH - 1) / PLAN_CH;
    if (nb > 0) plan_hist_kernel<<<nb, 256, 0, s>>>(p, hist);
    plan_scan_kernel<<<1, 1024, 0, s>>>(p, hist, nb, tiles, max_tiles);
    plan_scatter_kernel<<<nb > 0 ? nb : 1, 256, 0, s>>>(p, hist, nb);
    OFB_CHECK_LAUNCH("plan");
    return OFB_OK;
}

// Shared-expert gates sigmoid(x . v), one warp per token (tolerance-level:
// the reference has no gate; any summation order).
__global__ void __launch_bounds__(256) shared_gate_kernel(const float *__restrict__ x,
                                                          const float *__restrict__ v, int T, int D,
                                                          float *__restrict__ gsc) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)t * D);
    const float4 *v4 = reinterpret_cast<const float4 *>(v);
    float z = 0.f;
    for (int i = lane; i < D / 4; i += 32) {
        const float4 a = __ldg(x4 + i), b = __ldg(v4 + i);
        z += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
    }
    z = warp_sum(z);
    if (lane == 0) gsc[t] = 1.0f / (1.0f + expf(-z));
}

// out = resid + g*y_shared + sum_a w_a y_a (model.c:1007, :1090, :1142 order).
__global__ void combine_kernel(LayerArgs a) {
    const size_t total = (size_t)a.T * a.D;
    const int TK = a.T * a.K;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / a.D), n = (int)(i - (size_t)t * a.D);
        float o = a.resid ? a.resid[i] : 0.f;
        if (a.has_shared) {
            float ys = a.y[(size_t)(TK + t) * a.D + n];
            o += a.shared_gate ? a.gsc[t] * ys : ys;
        }
        float r = 0.f;
        for (int k = 0; k < a.K; k++) {
            const int asg = t * a.K + k;
            const float w = a.w[asg];
            if (w < 1e-6f) continue;
            r += w * a.y[(size_t)asg * a.D + n];
        }
        a.out[i] = o + r;
    }
}

// ---- interleaved (reference-slice) layout ---------------------------------
// Element i of expert e's slice is linear element i*E+e (gguf.c:683-705);
// gate/up slices are [D][H] (index k*H+m), down [H][D] (index j*D+n),
// model.c:351-357. The shared expert's tensors are plain [D][H] / [H][D].
__global__ void __launch_bounds__(256) interleaved_up_kernel(LayerArgs a) {
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int TK = a.T * a.K;
    const int units = *a.n_slots * a.H;
    for (int unit = warp; unit < units; unit += nwarps) {
        const int u = unit / a.H, m = unit - u * a.H;
        const int e = a.slot_expert[u];
        const bool sh = (e == a.E);
        const uint8_t *G = sh ? a.gate_sh : a.gate;
        const uint8_t *U = sh ? a.up_sh : a.up;
        const uint64_t es = sh ? 1 : (uint64_t)a.E, eo = sh ? 0 : (uint64_t)e;
        const int s1 = a.slot_start[u + 1];
        for (int s = a.slot_start[u]; s < s1; s++) {
            const int asg = a.assign[s];
            const float *xt = a.x + (size_t)asg_token(asg, TK, a.K) * a.D;
            float gp = 0.f, up = 0.f;
            for (int k = lane; k < a.D; k += 32) {
                const uint64_t lin = ((uint64_t)k * a.H + m) * es + eo;
                const int pos = (int)(lin % QK);
                gp += xt[k] * q4k_one(G + (lin / QK) * Q4K_BYTES, pos);
                up += xt[k] * q4k_one(U + (lin / QK) * Q4K_BYTES, pos);
            }
            gp = warp_sum(gp);
            up = warp_sum(up);
            if (lane == 0) a.h[(size_t)asg * a.H + m] = silu_ref(gp) * up;
        }
    }
}

__global__ void __launch_bounds__(256) interleaved_down_kernel(LayerArgs a) {
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int units = *a.n_slots * a.D;
    for (int unit = warp; unit < units; unit += nwarps) {
        const int u = unit / a.D, n = unit - u * a.D;
        const int e = a.slot_expert[u];
        const bool sh = (e == a.E);
        const uint8_t *Dn = sh ? a.down_sh : a.down;
        const uint64_t es = sh ? 1 : (uint64_t)a.E, eo = sh ? 0 : (uint64_t)e;
        const int s1 = a.slot_start[u + 1];
        for (int s = a.slot_start[u]; s < s1; s++) {
            const int asg = a.assign[s];
            const float *hrow = a.h + (size_t)asg * a.H;
            float part = 0.f;
            for (int j = lane; j < a.H; j += 32) {
                const uint64_t lin = ((uint64_t)j * a.D + n) * es + eo;
                part += hrow[j] * q6k_one(Dn + (lin / QK) * Q6K_BYTES, (int)(lin % QK));
            }
            part = warp_sum(part);
            if (lane == 0) a.y[(size_t)asg * a.D + n] = part;
        }
    }
}

// ---- workspace -----------------------------------------------------------
static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

WorkspaceLayout workspace_layout(const ofb_moe_config *c, int max_tokens) {
    WorkspaceLayout L;
    const size_t T = (size_t)max_tokens, K = c->top_k, E = c->n_experts;
    const size_t A = T * K + T;  // routed + shared assignments
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
    // single-launch decode words first (their size depends on the shape only)
    L.fsync = take((5 + 16) * 4);
    L.fcand = take((2 * E + 1) * 8);
    L.fh = take((K + 1) * (size_t)c->hidden * 8);
    L.fused_bytes = off;
    L.logits = take(T * E * 4);
    L.idx = take(T * K * 4);
    L.w = take(T * K * 4);
    L.gsc = take(T * 4);
    L.n_slots = take(4);
    L.slot_expert = take((E + 1) * 4);
    L.slot_start = take((E + 2) * 4);
    L.assign = take(A * 4);
    L.phist = take(plan_hist_ints(max_tokens, (int)K, (int)E) * 4);
    // h / y (f32) serve the decode kernels (T <= gemv_max_tokens) and the
    // interleaved path; the tensor-core prefill path uses bf16 x and h instead
    const bool inter = c->layout == OFB_LAYOUT_INTERLEAVED;
    const size_t Tg = (size_t)gemv_max_tokens((int)K, (int)E);
    const size_t Td = inter ? T : (T < Tg ? T : Tg);
    const size_t Ad = Td * K + Td;
    L.h = take(Ad * (size_t)c->hidden * 4);
    L.y = take(Ad * (size_t)c->d_model * 4);
    // tensor-core buffers whenever a call may exceed the fixed decode size:
    // the layer itself above gemv_max_tokens, and one-expert runs over the
    // same tokens (ofb_moe_shared) above the decode-kernel limit
    const bool prefill = !inter && max_tokens > gemv_limit(c->hidden) && c->hidden <= PREFILL_MAX_H;
    L.xb = take(prefill ? A * (size_t)c->d_model * 2 : 0);
    L.hb = take(prefill ? A * (size_t)c->hidden * 2 : 0);
    L.tiles = take(prefill ? (1 + 3 * (size_t)prefill_max_tiles(max_tokens, K, E)) * 4 : 0);
    const size_t Tf = (size_t)(max_tokens < FAST_ROUTE_MAX_T ? max_tokens : FAST_ROUTE_MAX_T);
    // certified routing holds (L~, B) per (token, expert): every token on the
    // contiguous layout (the large-batch router too), else the decode sizes
    L.cand = take((inter ? Tf : T) * (E + 1) * 16);
    L.norms = take(inter ? 0 : (T + E) * (size_t)(c->d_model / 64) * 4);
    const size_t Ts = T > (size_t)FAST_ROUTE_MAX_T ? (T < (size_t)ROUTE_SPLIT_MAX_T ? T : ROUTE_SPLIT_MAX_T - 1) : 0;
    L.segsum = take(inter ? 0 : Ts * E * (size_t)(c->d_model / 64) * 4);
    L.xq = take((Tf > Td ? Tf : Td) * xq_stride(c->d_model));
    // route tickets [64] + [1], route stats [3], pad [1], down-combine tickets [D/4]
    // ... then the prefill error flag [1]
    L.counters_bytes = (FAST_ROUTE_MAX_T + 4 + c->d_model / DOWN_TICKET_ROWS + 1) * 4;
    L.counters = take(L.counters_bytes);
    L.total = off;
    L.gemv_tokens = Td;
    L.gemv_rows = Ad;
    L.prefill_rows = prefill ? A : 0;
    L.prefill_tiles = prefill ? (size_t)prefill_max_tiles(max_tokens, K, E) : 0;
    return L;
}

int check_config(const ofb_moe_config *c) {
    if (!c) { set_error("NULL config"); return OFB_EINVAL; }
    if (c->d_model <= 0 || c->d_model % QK || c->hidden <= 0 || c->hidden % QK) {
        set_error("d_model (%d) and hidden (%d) must be positive multiples of 256", c->d_model, c->hidden);
        return OFB_EINVAL;
    }
    if (c->hidden > MAX_DECODE_H) { set_error("hidden %d > %d unsupported", c->hidden, MAX_DECODE_H); return OFB_EUNSUPPORTED; }
    if (c->n_experts < 1 || c->n_experts > 1024) { set_error("n_experts %d not in [1,1024]", c->n_experts); return OFB_EINVAL; }
    if (c->top_k < 1 || c->top_k > 16 || c->top_k > c->n_experts) { set_error("top_k %d invalid", c->top_k); return OFB_EINVAL; }
    if (c->layout != OFB_LAYOUT_CONTIGUOUS && c->layout != OFB_LAYOUT_INTERLEAVED) { set_error("bad layout %d", c->layout); return OFB_EINVAL; }
    if (c->routing != OFB_ROUTE_FORWARD && c->routing != OFB_ROUTE_GET_ROUTING) { set_error("bad routing %d", c->routing); return OFB_EINVAL; }
    return OFB_OK;
}

int run_moe_layer(const ofb_moe_config *cfg, const ofb_moe_weights *wt, const float *x,
                  const float *resid, float *out, int T, uint32_t *idx_out, float *w_out,
                  uint8_t *base, const WorkspaceLayout &L, cudaStream_t s, cudaEvent_t *ev,
                  const uint32_t *given_idx, const float *given_w, const __nv_bfloat16 *x_bf16) {
    const int D = cfg->d_model, H = cfg->hidden, E = cfg->n_experts, K = cfg->top_k;
    auto mark = [&](int i) { if (ev) cudaEventRecord(ev[i], s); };
    mark(0);
    float *logits = (float *)(base + L.logits);
    uint32_t *idx = given_idx ? const_cast<uint32_t *>(given_idx) : idx_out ? idx_out : (uint32_t *)(base + L.idx);
    float *w = given_w ? const_cast<float *>(given_w) : w_out ? w_out : (float *)(base + L.w);
    const bool has_shared = wt->gate_shexp && wt->up_shexp && wt->down_shexp;
    PlanArgs p;
    p.idx = idx; p.w = w; p.T = T; p.K = K; p.E = E; p.D = D;
    p.has_shared = has_shared; p.shared_gate = cfg->shared_gate && wt->shexp_gate;
    p.x = x; p.gate_v = wt->shexp_gate;
    p.gsc = (float *)(base + L.gsc);
    p.n_slots = (int *)(base + L.n_slots);
    p.slot_expert = (int *)(base + L.slot_expert);
    p.slot_start = (int *)(base + L.slot_start);
    p.assign = (int *)(base + L.assign);
    int st;
    // the plan also lays out the tensor-core tiles when the layer goes there
    const bool tc_path = cfg->layout == OFB_LAYOUT_CONTIGUOUS && !use_gemv(T, K, E, H) && H <= PREFILL_MAX_H &&
                         (size_t)prefill_max_tiles(T, K, E) <= L.prefill_tiles;
    int *plan_tiles = tc_path ? (int *)(base + L.tiles) : nullptr;
    if (T == 1 && !given_idx && wt->router && cfg->layout == OFB_LAYOUT_CONTIGUOUS) {
        // decode batch 1: the whole layer in one launch when the shape fits
        const bool has_sh = wt->gate_shexp && wt->up_shexp && wt->down_shexp;
        const bool use_gate = has_sh && cfg->shared_gate && wt->shexp_gate;
        FusedPlan fp;
        if ((!use_gate || !(reinterpret_cast<uintptr_t>(wt->shexp_gate) & 15)) &&
            fused_plan(cfg, use_gate, has_sh, sm_count(), fp)) {
            int *ctr = (int *)(base + L.counters);
            st = launch_decode_fused(cfg, wt, x, resid, out, idx_out, w_out, fp,
                                     (unsigned long long *)(base + L.fcand), (unsigned long long *)(base + L.fh),
                                     (unsigned int *)(base + L.fsync), ctr + FAST_ROUTE_MAX_T + 1, s);
            if (st) return st;
            for (int i = 1; i <= 4; i++) mark(i);
            return OFB_OK;
        }
    }
    const bool fast = !given_idx && wt->router && cfg->layout == OFB_LAYOUT_CONTIGUOUS && T <= FAST_ROUTE_MAX_T;
    if (fast) {
        // one launch: certified routing, shared-expert gates, dispatch plan
        int *ctr = (int *)(base + L.counters);
        if ((st = launch_route_fast(wt->router, x, p.shared_gate ? wt->shexp_gate : nullptr, T, D, E, K,
                                    cfg->routing, cfg->renorm, (double2 *)(base + L.cand),
                                    ctr + FAST_ROUTE_MAX_T, ctr + FAST_ROUTE_MAX_T + 1, idx, w, p.gsc,
                                    use_gemv(T, K, E, H) ? base + L.xq : nullptr,
                                    &p, s)))
            return st;
        mark(1);
        mark(2);
    } else if (!given_idx && wt->router && cfg->layout == OFB_LAYOUT_CONTIGUOUS && E <= 256) {
        // large batches: certified routing from a bounded fp32 GEMM; the last
        // selection block builds the plan
        int *ctr = (int *)(base + L.counters);
        // the certify warps also compute the shared-expert gates
        if ((st = launch_route_fast_large(wt->router, x, p.has_shared && p.shared_gate ? p.gate_v : nullptr, p.gsc, T,
                                          D, E, K, cfg->routing, cfg->renorm,
                                          (double2 *)(base + L.cand), (float *)(base + L.norms),
                                          (float *)(base + L.segsum), (int *)(base + L.logits), ctr, ctr + FAST_ROUTE_MAX_T + 1, idx, w, s)))
            return st;
        mark(1);
        if ((st = launch_plan(p, (int *)(base + L.phist), plan_tiles, prefill_max_tiles(T, K, E), s))) return st;
        mark(2);
    } else {
        if (given_idx) {
            // routing supplied by the caller
        } else if (wt->router) {
            if ((st = launch_router_logits(cfg->layout, wt->router, x, T, D, E, logits, s))) return st;
            if ((st = launch_route_select(logits, T, E, K, cfg->routing, cfg->renorm, idx, w, s))) return st;
        } else if ((st = launch_route_uniform(T, K, idx, w, s))) {
            return st;
        }
        mark(1);
        if ((st = launch_plan(p, (int *)(base + L.phist), plan_tiles, prefill_max_tiles(T, K, E), s))) return st;
        if (p.has_shared && p.shared_gate)
            shared_gate_kernel<<<(T + 7) / 8, 256, 0, s>>>(x, p.gate_v, T, D, p.gsc);
        OFB_CHECK_LAUNCH("plan");
        mark(2);
    }

    LayerArgs a;
    a.T = T; a.D = D; a.H = H; a.E = E; a.K = K;
    a.has_shared = has_shared; a.shared_gate = p.shared_gate;
    a.x = x; a.resid = resid; a.out = out;
    a.gate = (const uint8_t *)wt->gate_exps; a.up = (const uint8_t *)wt->up_exps;
    a.down = (const uint8_t *)wt->down_exps;
    a.gate_sh = (const uint8_t *)wt->gate_shexp; a.up_sh = (const uint8_t *)wt->up_shexp;
    a.down_sh = (const uint8_t *)wt->down_shexp;
    a.idx = idx; a.w = w; a.gsc = p.gsc;
    a.n_slots = p.n_slots; a.slot_expert = p.slot_expert; a.slot_start = p.slot_start;
    a.assign = p.assign;
    a.h = (float *)(base + L.h);
    a.y = (float *)(base + L.y);

    const int max_slots = (T * K < E ? T * K : E) + 1;
    const int sms = sm_count();
    if (cfg->layout == OFB_LAYOUT_INTERLEAVED) {
        interleaved_up_kernel<<<grid_for((uint64_t)max_slots * H, 8, sms * 8), 256, 0, s>>>(a);
        mark(3);
        interleaved_down_kernel<<<grid_for((uint64_t)max_slots * D, 8, sms * 8), 256, 0, s>>>(a);
        combine_kernel<<<grid_for((uint64_t)T * D, 256, sms * 4), 256, 0, s>>>(a);
        OFB_CHECK_LAUNCH("interleaved layer");
        mark(4);
        return OFB_OK;
    }
    a.xb_in = x_bf16;
    if (x_bf16 && (use_gemv(T, K, E, H) || H > PREFILL_MAX_H)) {
        set_error("bf16 token rows need the tensor-core path (more than %d rows, hidden <= %d)",
                  gemv_limit(H), PREFILL_MAX_H);
        return OFB_EUNSUPPORTED;
    }
    if (use_gemv(T, K, E, H)) {
        if ((size_t)T > L.gemv_tokens || (size_t)T * K + (has_shared ? T : 0) > L.gemv_rows) {
            set_error("workspace holds %zu decode-path tokens; call needs %d", L.gemv_tokens, T);
            return OFB_ETOOLARGE;
        }
        unsigned char *xq = base + L.xq;
        if (!fast && (st = launch_quantize_x(x, T, D, xq, s))) return st;
        if ((st = launch_up_q(a, xq, max_slots, s))) return st;
        mark(3);
        int *tickets = (int *)(base + L.counters) + FAST_ROUTE_MAX_T + 4;
        if ((st = launch_down_q(a, tickets, max_slots, s))) return st;
        mark(4);
        return OFB_OK;
    }
    // prefill-sized batches: tcgen05 grouped GEMMs (prefill.cu)
    if (H > PREFILL_MAX_H) {
        set_error("batches above %d tokens need hidden <= %d (got %d)", gemv_max_tokens(K, E), PREFILL_MAX_H, H);
        return OFB_EUNSUPPORTED;
    }
    if ((size_t)T * K + T > L.prefill_rows || (size_t)prefill_max_tiles(T, K, E) > L.prefill_tiles) {
        set_error("workspace has no tensor-core buffers for %d tokens (rows %zu, tiles %zu)", T, L.prefill_rows,
                  L.prefill_tiles);
        return OFB_ETOOLARGE;
    }
    int *err = (int *)(base + L.counters) + FAST_ROUTE_MAX_T + 4 + D / DOWN_TICKET_ROWS;
    if ((st = launch_prefill(a, x, p.n_slots, (__nv_bfloat16 *)(base + L.xb), (__nv_bfloat16 *)(base + L.hb),
                             (int *)(base + L.tiles), !fast && plan_tiles != nullptr, err, s, ev ? ev[2] : nullptr, ev ? ev[3] : nullptr)))
        return st;
    mark(4);
    return OFB_OK;
}

}  // namespace ofb

using namespace ofb;


extern "C" size_t ofb_workspace_size(const ofb_moe_config *cfg, int max_tokens) {
    if (check_config(cfg) || max_tokens < 1) return 0;
    return workspace_layout(cfg, max_tokens).total;
}

extern "C" int ofb_workspace_create(const ofb_moe_config *cfg, int max_tokens, ofb_workspace **ws) {
    int st = check_config(cfg);
    if (st) return st;
    if (!ws || max_tokens < 1) { set_error("workspace_create: bad arguments"); return OFB_EINVAL; }
    ofb_workspace *w = (ofb_workspace *)calloc(1, sizeof(ofb_workspace));
    if (!w) { set_error("workspace_create: host OOM"); return OFB_ENOMEM; }
    w->cfg = *cfg;
    w->max_tokens = max_tokens;
    w->layout = workspace_layout(cfg, max_tokens);
    cudaError_t e = cudaMalloc((void **)&w->base, w->layout.total);
    if (e != cudaSuccess) { free(w); return cuda_status(e, "workspace cudaMalloc"); }
    // routing tickets must start at zero (each call leaves them at zero); the
    // single-launch decode's epoch and tagged words start at zero once
    e = cudaMemset(w->base + w->layout.counters, 0, w->layout.counters_bytes);
    if (e == cudaSuccess) e = cudaMemset(w->base, 0, w->layout.fused_bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { cudaFree(w->base); free(w); return cuda_status(e, "workspace init"); }
    *ws = w;
    return OFB_OK;
}

extern "C" int ofb_workspace_destroy(ofb_workspace *ws) {
    if (!ws) return OFB_OK;
    cudaError_t e = cudaFree(ws->base);
    free(ws);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "workspace cudaFree");
}

int ofb::check_ws(const ofb_moe_config *cfg, const ofb_workspace *ws, int T) {
    if (!ws) { set_error("NULL workspace"); return OFB_EINVAL; }
    if (T > ws->max_tokens) { set_error("n_tokens %d > workspace max_tokens %d", T, ws->max_tokens); return OFB_ETOOLARGE; }
    const ofb_moe_config &c = ws->cfg;
    if (c.d_model != cfg->d_model || c.hidden != cfg->hidden || c.n_experts != cfg->n_experts ||
        c.top_k != cfg->top_k || c.layout != cfg->layout) {
        set_error("workspace was created for a different layer shape");
        return OFB_EINVAL;
    }
    return OFB_OK;
}

extern "C" int ofb_route(const ofb_moe_config *cfg, const float *router, const float *x,
                         int n_tokens, uint32_t *idx, float *w, ofb_workspace *ws, void *stream) {
    int st = check_config(cfg);
    if (st) return st;
    if (!x || !idx || !w || n_tokens < 0) { set_error("ofb_route: bad arguments"); return OFB_EINVAL; }
    if ((st = check_ws(cfg, ws, n_tokens))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!router) return launch_route_uniform(n_tokens, cfg->top_k, idx, w, s);
    float *logits = (float *)(ws->base + ws->layout.logits);
    if ((st = launch_router_logits(cfg->layout, router, x, n_tokens, cfg->d_model, cfg->n_experts, logits, s))) return st;
    return launch_route_select(logits, n_tokens, cfg->n_experts, cfg->top_k, cfg->routing, cfg->renorm, idx, w, s);
}

extern "C" int ofb_route_certified(const ofb_moe_config *cfg, const float *router, const float *x,
                                   int n_tokens, uint32_t *idx, float *w, ofb_workspace *ws, void *stream) {
    int st = check_config(cfg);
    if (st) return st;
    if (!x || !idx || !w || n_tokens < 0) { set_error("ofb_route_certified: bad arguments"); return OFB_EINVAL; }
    if ((st = check_ws(cfg, ws, n_tokens))) return st;
    if (n_tokens == 0) return OFB_OK;
    if (!router || cfg->layout != OFB_LAYOUT_CONTIGUOUS || cfg->n_experts > 256)
        return ofb_route(cfg, router, x, n_tokens, idx, w, ws, stream);
    if ((reinterpret_cast<uintptr_t>(router) | reinterpret_cast<uintptr_t>(x)) & 15) {
        set_error("ofb_route_certified: router and x must be 16-byte aligned");
        return OFB_EINVAL;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const WorkspaceLayout &L = ws->layout;
    int *ctr = (int *)(ws->base + L.counters);
    const int D = cfg->d_model, E = cfg->n_experts, K = cfg->top_k;
    if (n_tokens <= FAST_ROUTE_MAX_T)
        return launch_route_fast(router, x, nullptr, n_tokens, D, E, K, cfg->routing, cfg->renorm,
                                 (double2 *)(ws->base + L.cand), ctr + FAST_ROUTE_MAX_T, ctr + FAST_ROUTE_MAX_T + 1,
                                 idx, w, (float *)(ws->base + L.gsc), nullptr, nullptr, s);
    return launch_route_fast_large(router, x, nullptr, nullptr, n_tokens, D, E, K, cfg->routing, cfg->renorm,
                                   (double2 *)(ws->base + L.cand), (float *)(ws->base + L.norms),
                                   (float *)(ws->base + L.segsum), (int *)(ws->base + L.logits), ctr, ctr + FAST_ROUTE_MAX_T + 1, idx, w, s);
}

extern "C" int ofb_moe_forward(const ofb_moe_config *cfg, const ofb_moe_weights *w,
                               const float *x, const float *resid, float *out, int n_tokens,
                               uint32_t *idx_out, float *w_out, ofb_workspace *ws, void *stream) {
    int st = check_config(cfg);
    if (st) return st;
    if (!w || n_tokens < 0) { set_error("ofb_moe_forward: bad arguments"); return OFB_EINVAL; }
    if ((st = check_ws(cfg, ws, n_tokens))) return st;
    if (n_tokens == 0) return OFB_OK;
    if (!x || !out) { set_error("ofb_moe_forward: NULL activations"); return OFB_EINVAL; }
    if (!w->gate_exps || !w->up_exps || !w->down_exps) { set_error("ofb_moe_forward: NULL expert tensor"); return OFB_EINVAL; }
    if ((reinterpret_cast<uintptr_t>(w->gate_exps) | reinterpret_cast<uintptr_t>(w->up_exps) |
         reinterpret_cast<uintptr_t>(w->down_exps) | reinterpret_cast<uintptr_t>(w->gate_shexp) |
         reinterpret_cast<uintptr_t>(w->up_shexp) | reinterpret_cast<uintptr_t>(w->down_shexp) |
         reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w->router)) & 15) {
        set_error("ofb_moe_forward: tensors must be 16-byte aligned");
        return OFB_EINVAL;
    }
    return run_moe_layer(cfg, w, x, resid, out, n_tokens, idx_out, w_out, ws->base, ws->layout,
                         static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int ofb_moe_forward_profiled(const ofb_moe_config *cfg, const ofb_moe_weights *w,
                                        const float *x, const float *resid, float *out,
                                        int n_tokens, ofb_workspace *ws, void *stream,
                                        float *phase_ms) {
    int st = check_config(cfg);
    if (st) return st;
    if (!w || !x || !out || !phase_ms || n_tokens < 1) { set_error("profiled: bad arguments"); return OFB_EINVAL; }
    if ((st = check_ws(cfg, ws, n_tokens))) return st;
    cudaEvent_t ev[5];
    for (int i = 0; i < 5; i++)
        if (cudaEventCreate(&ev[i]) != cudaSuccess) return cuda_status(cudaGetLastError(), "event create");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = run_moe_layer(cfg, w, x, resid, out, n_tokens, nullptr, nullptr, ws->base, ws->layout, s, ev);
    if (!st) {
        cudaError_t e = cudaEventSynchronize(ev[4]);
        if (e != cudaSuccess) st = cuda_status(e, "profiled sync");
        for (int i = 0; !st && i < 4; i++) cudaEventElapsedTime(&phase_ms[i], ev[i], ev[i + 1]);
    }
    for (int i = 0; i < 5; i++) cudaEventDestroy(ev[i]);
    return st;
}

// Row metadata {local expert, float bits of weight} -> idx / w arrays.
__global__ void unpack_meta_kernel(const int32_t *__restrict__ meta, int n, uint32_t *__restrict__ idx,
                                   float *__restrict__ w) {
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
        idx[r] = (uint32_t)meta[2 * r];
        w[r] = __int_as_float(meta[2 * r + 1]);
    }
}

__global__ void fill_kernel(float *__restrict__ p, int n, float v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int ofb::run_experts_given(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x_rows,
                      const __nv_bfloat16 *x_rows_bf16, int n_rows, const int32_t *row_meta, float *out_rows,
                      ofb_workspace *ws, cudaStream_t s) {
    ofb_moe_weights routed = *w;  // routed experts only
    routed.router = nullptr;
    routed.gate_shexp = routed.up_shexp = routed.down_shexp = nullptr;
    routed.shexp_gate = nullptr;
    uint32_t *idx = (uint32_t *)(ws->base + ws->layout.idx);
    float *wt = (float *)(ws->base + ws->layout.w);
    unpack_meta_kernel<<<grid_for((size_t)n_rows, 256, 148 * 4), 256, 0, s>>>(row_meta, n_rows, idx, wt);
    OFB_CHECK_LAUNCH("unpack row metadata");
    // rows whose weight is below the skip threshold get no expert term; on
    // the decode-sized path the combine writes rows only when some row has
    // one, so start from zeros (the tensor-core path initialises out itself)
    if (use_gemv(n_rows, 1, cfg->n_experts, cfg->hidden)) {
        cudaError_t e = cudaMemsetAsync(out_rows, 0, (size_t)n_rows * cfg->d_model * sizeof(float), s);
        if (e != cudaSuccess) return cuda_status(e, "ofb_moe_experts memset");
    }
    return run_moe_layer(cfg, &routed, x_rows, nullptr, out_rows, n_rows, nullptr, nullptr, ws->base, ws->layout,
                         s, nullptr, idx, wt, x_rows_bf16);
}

extern "C" int ofb_moe_experts(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x_rows,
                               int n_rows, const int32_t *row_meta, float *out_rows, ofb_workspace *ws,
                               void *stream) {
    int st = check_config(cfg);
    if (st) return st;
    if (!w || n_rows < 0) { set_error("ofb_moe_experts: bad arguments"); return OFB_EINVAL; }
    if (cfg->top_k != 1 || cfg->layout != OFB_LAYOUT_CONTIGUOUS) {
        set_error("ofb_moe_experts: needs top_k = 1 and the contiguous layout");
        return OFB_EINVAL;
    }
    if ((st = check_ws(cfg, ws, n_rows))) return st;
    if (n_rows == 0) return OFB_OK;
    if (!x_rows || !row_meta || !out_rows || !w->gate_exps || !w->up_exps || !w->down_exps) {
        set_error("ofb_moe_experts: NULL pointer");
        return OFB_EINVAL;
    }
    if (!aligned16(x_rows) || !aligned16(w->gate_exps) || !aligned16(w->up_exps) || !aligned16(w->down_exps)) {
        set_error("ofb_moe_experts: tensors must be 16-byte aligned");
        return OFB_EINVAL;
    }
    return run_experts_given(cfg, w, x_rows, nullptr, n_rows, row_meta, out_rows, ws,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int ofb_moe_shared(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x,
                              const float *resid, float *out, int n_tokens, ofb_workspace *ws, void *stream) {
    int st = check_config(cfg);
    if (st) return st;
    if (!w || !ws || n_tokens < 0) { set_error("ofb_moe_shared: bad arguments"); return OFB_EINVAL; }
    if (n_tokens == 0) return OFB_OK;
    if (!x || !out || !w->gate_shexp || !w->up_shexp || !w->down_shexp) {
        set_error("ofb_moe_shared: NULL pointer");
        return OFB_EINVAL;
    }
    const ofb_moe_config &wc = ws->cfg;
    if (wc.d_model != cfg->d_model || wc.hidden != cfg->hidden || wc.layout != OFB_LAYOUT_CONTIGUOUS ||
        cfg->layout != OFB_LAYOUT_CONTIGUOUS || n_tokens > ws->max_tokens) {
        set_error("ofb_moe_shared: workspace does not fit (shape, contiguous layout, max_tokens)");
        return OFB_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w->gate_shexp) || !aligned16(w->up_shexp) || !aligned16(w->down_shexp)) {
        set_error("ofb_moe_shared: tensors must be 16-byte aligned");
        return OFB_EINVAL;
    }
    // the shared expert as a one-expert layer: every token routed to it with
    // weight g_t (a workspace of any expert count / top_k >= 1 holds this);
    // the routed skip rule then drops a term whose gate is below 1e-6, a
    // change below 1e-6 of |y|
    ofb_moe_config one = *cfg;
    one.n_experts = 1;
    one.top_k = 1;
    ofb_moe_weights sw = {};
    sw.gate_exps = w->gate_shexp;
    sw.up_exps = w->up_shexp;
    sw.down_exps = w->down_shexp;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t *idx = (uint32_t *)(ws->base + ws->layout.idx);
    float *g = (float *)(ws->base + ws->layout.w);
    cudaError_t e = cudaMemsetAsync(idx, 0, (size_t)n_tokens * sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "ofb_moe_shared memset");
    if (cfg->shared_gate && w->shexp_gate)
        shared_gate_kernel<<<(n_tokens + 7) / 8, 256, 0, s>>>(x, w->shexp_gate, n_tokens, cfg->d_model, g);
    else
        fill_kernel<<<grid_for((size_t)n_tokens, 256, 148), 256, 0, s>>>(g, n_tokens, 1.0f);
    OFB_CHECK_LAUNCH("shared gates");
    return run_moe_layer(&one, &sw, x, resid, out, n_tokens, nullptr, nullptr, ws->base, ws->layout, s, nullptr,
                         idx, g);
}

extern "C" int ofb_workspace_route_stats(ofb_workspace *ws, int counts[3]) {
    if (!ws || !counts) { set_error("route_stats: NULL argument"); return OFB_EINVAL; }
    cudaError_t e = cudaMemcpy(counts, ws->base + ws->layout.counters + (FAST_ROUTE_MAX_T + 1) * 4,
                               3 * sizeof(int), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "route_stats copy");
}

extern "C" int ofb_workspace_device_errors(ofb_workspace *ws, unsigned *bits) {
    if (!ws || !bits) { set_error("device_errors: NULL argument"); return OFB_EINVAL; }
    const WorkspaceLayout &L = ws->layout;
    const int D = ws->cfg.d_model;
    unsigned fused = 0;
    int prefill = 0;
    unsigned *fw = (unsigned *)(ws->base + L.fsync) + 2;
    int *pf = (int *)(ws->base + L.counters) + FAST_ROUTE_MAX_T + 4 + D / DOWN_TICKET_ROWS;
    cudaError_t e = cudaMemcpy(&fused, fw, sizeof(fused), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&prefill, pf, sizeof(prefill), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(fw, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(pf, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "device_errors copy");
    *bits = (fused & 3u) | (prefill ? 4u : 0u);
    return OFB_OK;
}
