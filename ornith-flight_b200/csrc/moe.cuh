// moe.cuh — internal structures of the MoE layer kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

#include "ornith_moe.h"

namespace ofb {

struct PlanArgs {
    const uint32_t *idx;
    const float *w;
    int T, K, E, D;
    int has_shared, shared_gate;
    const float *x, *gate_v;
    float *gsc;
    int *n_slots, *slot_expert, *slot_start, *assign;
};

struct LayerArgs {
    int T, D, H, E, K;
    int has_shared, shared_gate;
    const float *x;
    const float *resid;
    float *out;
    const uint8_t *gate, *up, *down;
    const uint8_t *gate_sh, *up_sh, *down_sh;
    const uint32_t *idx;
    const float *w, *gsc;
    const int *n_slots, *slot_expert, *slot_start, *assign;
    float *h, *y;
    const __nv_bfloat16 *xb_in;  // token rows already bf16 (tensor-core path only), else NULL
};

// Byte offsets of the scratch regions inside one workspace allocation.
struct WorkspaceLayout {
    // single-launch decode (T = 1): epoch / finished / error words, tagged
    // (L~, B) per expert + shared gate, tagged h per top-k slot + shared
    // expert. First in the workspace at a size that depends only on the layer
    // shape, so a fixed scratch keeps it in place across calls of any size.
    size_t fsync, fcand, fh, fused_bytes;
    size_t logits, idx, w, gsc, n_slots, slot_expert, slot_start, assign, h, y;
    size_t phist;     // per-CTA expert counts of the many-CTA plan (plan_hist_ints)
    size_t cand;      // fast routing: (approximate logit, bound) per (token, row)
    size_t norms;     // large-batch routing: segment norms of x rows and router rows
    size_t segsum;    // large-batch routing below ROUTE_SPLIT_MAX_T tokens: segment sums [seg][token][expert]
    size_t xq;        // decode: quantised activations [T][xq_stride(D)]
    size_t xb, hb;    // prefill: bf16 x rows [A][D] and h rows [A][H], both in slot order
    size_t tiles;     // prefill: tile count + (slot, start, n) per tile
    size_t counters;  // fast routing tickets [T] + [1] and stats [3]; zero at creation
    size_t counters_bytes;
    size_t total;
    // capacities the regions were sized for (checked before every launch)
    size_t gemv_tokens;    // tokens h / y / xq hold on the decode-kernel path
    size_t gemv_rows;      // assignments (incl. shared) h / y hold
    size_t prefill_rows;   // assignments xb / hb hold (0: no tensor-core path)
    size_t prefill_tiles;  // tile-list entries
};

// Token counts up to which routing uses the certified fast kernel.
constexpr int FAST_ROUTE_MAX_T = 64;
// Decode expert kernels (decode.cu): token and hidden-width limits.
constexpr int MAX_DECODE_T = 32;
constexpr int MAX_DECODE_H = 1024;
// Output rows per completion ticket of the decode down kernel.
constexpr int DOWN_TICKET_ROWS = 4;
// Tensor-core prefill kernels: the down kernel holds 128 Q6_K rows in shared memory.
constexpr int PREFILL_MAX_H = 512;
// Batches the dp4a decode kernels take: up to 4 tokens when the tensor-core
// kernels can take over (hidden <= PREFILL_MAX_H), up to MAX_DECODE_T
// otherwise. Measured on the 2048 x 512, 256-expert layer (us per layer,
// decode kernels / tensor-core kernels): 8 tokens 135 / 114, 16 tokens 240 /
// 158, 32 tokens 381 / 233; at 4 tokens they tie.
constexpr int GEMV_T_WITH_TC = 4;
__host__ __device__ inline int gemv_limit(int H) { return H <= PREFILL_MAX_H ? GEMV_T_WITH_TC : MAX_DECODE_T; }
__host__ __device__ inline int gemv_max_tokens(int, int) { return MAX_DECODE_T; }  // decode buffer sizing
__host__ __device__ inline bool use_gemv(int T, int K, int E, int H) {
    return H <= MAX_DECODE_H && T <= gemv_limit(H);
}

int launch_quantize_x(const float *x, int T, int D, unsigned char *xq, cudaStream_t s);
int prefill_max_tiles(int T, int K, int E);
constexpr int PF_NMAX = 192;  // token rows per tensor-core tile (the MMA's N, at most)
// Dispatch plan over many CTAs (large batches): per-CTA histograms, one
// scan block (slots, and the tensor-core tile list when `tiles` is given),
// then the scatter. `hist` holds plan_hist_ints(T, K, E) ints.
constexpr int PLAN_CH = 256;  // routed assignments per histogram CTA
inline size_t plan_hist_ints(int T, int K, int E) {
    const size_t nb = ((size_t)T * K + PLAN_CH - 1) / PLAN_CH;
    return (nb + 1) * (size_t)E + 1;
}
int launch_plan(const PlanArgs &p, int *hist, int *tiles, int max_tiles, cudaStream_t s);
int launch_prefill(const LayerArgs &la, const float *x, int *n_slots, __nv_bfloat16 *xb, __nv_bfloat16 *hb,
                   int *tiles, bool tiles_ready, int *err, cudaStream_t s, cudaEvent_t before = nullptr,
                   cudaEvent_t between = nullptr);
int launch_up_q(const LayerArgs &a, const unsigned char *xq, int max_slots, cudaStream_t s);
int launch_down_q(const LayerArgs &a, int *tickets, int max_slots, cudaStream_t s);

// Certified routing for batches above FAST_ROUTE_MAX_T: fp32 GEMM logits with
// rigorous bounds, the same per-token certificate (one warp per token), exact
// fallback for the tokens it leaves (flagged list, T ints; *n_flagged is
// scratch). norms: scratch of (T + E) * d_model / 64 floats.
int launch_route_fast_large(const float *W, const float *x, const float *gate_v, float *gsc, int T, int D, int E,
                            int K, int routing, int renorm, double2 *cand, float *norms, float *segsum, int *flagged, int *n_flagged, int *stats,
                            uint32_t *idx, float *w, cudaStream_t s);
// Tokens below which the large-batch router splits its GEMM over segments
// (segsum holds T * E * d_model / 64 floats for those batches).
constexpr int ROUTE_SPLIT_MAX_T = 1024;
int launch_route_fast(const float *W, const float *x, const float *gate_v, int T, int D, int E, int K,
                      int routing, int renorm, double2 *cand, int *all_cnt, int *stats,
                      uint32_t *idx, float *w, float *gsc, unsigned char *xq, const PlanArgs *plan,
                      cudaStream_t s);

// Quantised activations of one token: int8 xh[D], uint8 xl[D], then per
// 32-element sub-block the f32 scale s and the f32 sum of x.
__host__ __device__ inline size_t xq_stride(int D) { return (size_t)2 * D + (size_t)8 * (D / 32); }

// Shared-memory plan of the single-launch decode kernel (decode_fused.cu):
// per-CTA share sizes and region offsets, identical on host and device.
struct FusedPlan {
    int G, rmax, upc, ngc, dg;
    uint32_t upb;  // bytes of the gate-row region (the up rows follow)
    uint32_t sdn;  // bytes of one slot's down slab (ngc output rows + alignment)
    uint32_t o_x, o_xq, o_rr, o_dn, o_up, o_hb, o_part, o_hst, o_hq, o_sel, o_ys, o_res, o_bar, total;
};
bool fused_plan(const ofb_moe_config *cfg, bool use_gate, bool has_shared, int grid, FusedPlan &p);

// Work shares of the single-launch decode kernel in 16-row h groups (one Q6_K
// scale group of h each): CTA c computes routed groups [rg0, rg1) of the
// K * H / 16 (pairs 16 * rg0 .. 16 * rg1 in top-k slot order) and, if it has
// the fewest routed groups, shared-expert groups [sg0, sg1) of H / 16, so
// every group is quantised by the CTA that computed it.
struct FdShare { int rg0, rg1, sg0, sg1; };
__host__ __device__ inline FdShare fd_share(int c, int G, int NR, int NS) {
    FdShare s;
    s.rg0 = (int)((long long)c * NR / G);
    s.rg1 = (int)((long long)(c + 1) * NR / G);
    s.sg0 = s.sg1 = 0;
    const int q = NR / G, L = G - NR % G;  // L CTAs have q routed groups
    if (s.rg1 - s.rg0 == q) {
        const int j = c * (1 + q) - s.rg0;  // rank among them
        s.sg0 = (int)((long long)j * NS / L);
        s.sg1 = (int)((long long)(j + 1) * NS / L);
    }
    return s;
}
int launch_decode_fused(const ofb_moe_config *cfg, const ofb_moe_weights *wt, const float *x, const float *resid,
                        float *out, uint32_t *idx_out, float *w_out, const FusedPlan &plan,
                        unsigned long long *cand, unsigned long long *hll, unsigned int *sync, int *stats,
                        cudaStream_t s);

WorkspaceLayout workspace_layout(const ofb_moe_config *c, int max_tokens);
int check_config(const ofb_moe_config *c);
// given_idx / given_w (device, [T][top_k]): routing supplied by the caller;
// the router is skipped and the layer runs from the dispatch plan on.
int run_moe_layer(const ofb_moe_config *cfg, const ofb_moe_weights *wt, const float *x,
                  const float *resid, float *out, int T, uint32_t *idx_out, float *w_out,
                  uint8_t *base, const WorkspaceLayout &L, cudaStream_t s,
                  cudaEvent_t *phase_events /* 5 events or NULL */,
                  const uint32_t *given_idx = nullptr, const float *given_w = nullptr,
                  const __nv_bfloat16 *x_bf16 = nullptr);

}  // namespace ofb

// A workspace: the scratch of one layer shape for up to max_tokens tokens.
struct ofb_workspace {
    ofb_moe_config cfg;
    int max_tokens;
    uint8_t *base;
    ofb::WorkspaceLayout layout;
};

namespace ofb {
int check_ws(const ofb_moe_config *cfg, const ofb_workspace *ws, int T);
// Routed experts over rows with given (local expert, weight) metadata; the
// rows are f32 (x_rows) or, on the tensor-core path, bf16 (x_rows_bf16).
int run_experts_given(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x_rows,
                      const __nv_bfloat16 *x_rows_bf16, int n_rows, const int32_t *row_meta, float *out_rows,
                      ofb_workspace *ws, cudaStream_t s);
}  // namespace ofb
