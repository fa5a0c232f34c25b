/*
 * moe.c — CPU restatement of ornith-flight's MoE feed-forward block.
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker, never the product.
 *
 * Follows engine/src/model.c:992-1143 (router GEMV, softmax over all
 * experts, partial exchange sort, per-expert SwiGLU, weighted combine,
 * residual adds) and model.c:264-321 (model_get_routing variant). All sums
 * are sequential fp32 with the reference's operand order; expf is glibc's.
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

float orc_expf(float x) { return expf(x); }

void orc_expf_batch(const float *x, float *out, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) out[i] = expf(x[i]);
}

/* engine/src/model.c:340-344 */
float orc_silu(float x) {
    if (x < -50.0f) return 0.0f;
    if (x > 50.0f) return x;
    return x / (1.0f + expf(-x));
}

/* engine/src/gpu.c:104-115 */
void orc_matmul(float *C, const float *A, const float *B, int M, int N, int K) {
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            float s = 0.0f;
            for (int k = 0; k < K; k++) s += A[i * K + k] * B[k * N + j];
            C[i * N + j] = s;
        }
}

/* Partial exchange sort of the first k positions (model.c:1042-1049 and the
 * full sort of model.c:299-302 agree on the first k positions): position i
 * takes any later element that is strictly greater, swapping it out. */
static void exchange_topk(float *val, int *idx, int n, int k) {
    for (int i = 0; i < k; i++)
        for (int j = i + 1; j < n; j++)
            if (val[j] > val[i]) {
                float tv = val[i]; val[i] = val[j]; val[j] = tv;
                int ti = idx[i]; idx[i] = idx[j]; idx[j] = ti;
            }
}

static float router_logit(const orc_moe_cfg *c, const float *x, const float *W, int e) {
    float s = 0.0f;
    if (c->layout == ORC_LAYOUT_INTERLEAVED) {
        /* model.c:1019-1025: W[d*E+e] */
        for (int d = 0; d < c->d_model; d++) s += x[d] * W[(size_t)d * c->n_experts + e];
    } else {
        /* [E][D] rows: same summation order over d */
        for (int d = 0; d < c->d_model; d++) s += x[d] * W[(size_t)e * c->d_model + d];
    }
    return s;
}

void orc_route_token(const orc_moe_cfg *c, const float *x, const float *W,
                     uint32_t *idx_out, float *w_out) {
    int E = c->n_experts, k = c->top_k;
    if (!W) { /* model.c:283-289: uniform fallback on experts 0..k-1 */
        for (int a = 0; a < k; a++) { idx_out[a] = (uint32_t)a; w_out[a] = 1.0f / k; }
        return;
    }
    float *val = (float *)malloc(sizeof(float) * E);
    int *idx = (int *)malloc(sizeof(int) * E);
    for (int e = 0; e < E; e++) { val[e] = router_logit(c, x, W, e); idx[e] = e; }
    if (c->routing == ORC_ROUTE_GET_ROUTING) {
        /* model.c:292-317: sort logits, softmax over the top-k logits */
        exchange_topk(val, idx, E, k);
        float mx = val[0], sum = 0.0f;
        for (int a = 0; a < k; a++) { float s = expf(val[a] - mx); w_out[a] = s; sum += s; }
        for (int a = 0; a < k; a++) { w_out[a] /= sum; idx_out[a] = (uint32_t)idx[a]; }
    } else {
        /* model.c:1027-1049: softmax over all experts, then select */
        float mx = val[0];
        for (int e = 1; e < E; e++) if (val[e] > mx) mx = val[e];
        float sum = 0.0f;
        for (int e = 0; e < E; e++) { val[e] = expf(val[e] - mx); sum += val[e]; }
        for (int e = 0; e < E; e++) val[e] /= sum;
        exchange_topk(val, idx, E, k);
        float ssum = 0.0f;
        for (int a = 0; a < k; a++) ssum += val[a];
        for (int a = 0; a < k; a++) {
            idx_out[a] = (uint32_t)idx[a];
            w_out[a] = c->renorm ? val[a] / ssum : val[a];
        }
    }
    free(val);
    free(idx);
}

/* Dequantised expert matrices, laid out so that
 *   gate/up: contiguous => [H][D] (row m, K fastest); interleaved => [D][H]
 *   down:    contiguous => [D][H];                    interleaved => [H][D] */
typedef struct { float *g, *u, *dn; } expert_f32;

/* Dequant used by the layer: the restatement by default; orc_set_dequant()
 * swaps in the reference's own compiled gguf.c (oracle/_ref) for timing. */
static orc_tensor_fn g_tensor_fn = orc_dequant_tensor;
static orc_slice_fn g_slice_fn = orc_dequant_slice;

void orc_set_dequant(orc_tensor_fn t, orc_slice_fn s) {
    g_tensor_fn = t ? t : orc_dequant_tensor;
    g_slice_fn = s ? s : orc_dequant_slice;
}

static int load_expert(const orc_moe_cfg *c, const orc_moe_weights *wt, int e, expert_f32 *x) {
    size_t HD = (size_t)c->hidden * c->d_model;
    x->g = (float *)malloc(HD * 4);
    x->u = (float *)malloc(HD * 4);
    x->dn = (float *)malloc(HD * 4);
    if (!x->g || !x->u || !x->dn) return 0;
    if (e < 0) { /* shared expert: whole-tensor decode (model.c:846-853) */
        return g_tensor_fn(wt->gate_shexp, ORC_TYPE_Q4_K, HD, x->g) &&
               g_tensor_fn(wt->up_shexp, ORC_TYPE_Q4_K, HD, x->u) &&
               g_tensor_fn(wt->down_shexp, ORC_TYPE_Q6_K, HD, x->dn);
    }
    if (c->layout == ORC_LAYOUT_INTERLEAVED) {
        uint64_t n = (uint64_t)HD * c->n_experts;
        return g_slice_fn(wt->gate_exps, ORC_TYPE_Q4_K, n, c->n_experts, e, x->g) &&
               g_slice_fn(wt->up_exps, ORC_TYPE_Q4_K, n, c->n_experts, e, x->u) &&
               g_slice_fn(wt->down_exps, ORC_TYPE_Q6_K, n, c->n_experts, e, x->dn);
    }
    size_t nb = HD / ORC_QK;
    const uint8_t *g = (const uint8_t *)wt->gate_exps + (size_t)e * nb * ORC_Q4K_BYTES;
    const uint8_t *u = (const uint8_t *)wt->up_exps + (size_t)e * nb * ORC_Q4K_BYTES;
    const uint8_t *d = (const uint8_t *)wt->down_exps + (size_t)e * nb * ORC_Q6K_BYTES;
    return g_tensor_fn(g, ORC_TYPE_Q4_K, HD, x->g) &&
           g_tensor_fn(u, ORC_TYPE_Q4_K, HD, x->u) &&
           g_tensor_fn(d, ORC_TYPE_Q6_K, HD, x->dn);
}

static void free_expert(expert_f32 *x) { free(x->g); free(x->u); free(x->dn); }

/* SwiGLU of one token through one dequantised expert (model.c:1085-1088 with
 * cpu_matmul_vec model.c:351-357: sequential fp32 over the input index). */
static void expert_apply(const orc_moe_cfg *c, const expert_f32 *m, const float *x, float *y,
                         float *hbuf) {
    int D = c->d_model, H = c->hidden;
    int rowmajor = (c->layout == ORC_LAYOUT_CONTIGUOUS);
    for (int j = 0; j < H; j++) {
        float g = 0.0f, u = 0.0f;
        for (int k = 0; k < D; k++) {
            size_t o = rowmajor ? (size_t)j * D + k : (size_t)k * H + j;
            g += x[k] * m->g[o];
        }
        for (int k = 0; k < D; k++) {
            size_t o = rowmajor ? (size_t)j * D + k : (size_t)k * H + j;
            u += x[k] * m->u[o];
        }
        hbuf[j] = orc_silu(g) * u;
    }
    for (int n = 0; n < D; n++) {
        float s = 0.0f;
        for (int j = 0; j < H; j++) {
            size_t o = rowmajor ? (size_t)n * H + j : (size_t)j * D + n;
            s += hbuf[j] * m->dn[o];
        }
        y[n] = s;
    }
}

int orc_moe_forward(const orc_moe_cfg *c, const orc_moe_weights *wt,
                    const float *x, const float *resid, int T, float *out,
                    uint32_t *idx_out, float *w_out) {
    if (!c || !wt || !x || !out || T < 0) return 0;
    int D = c->d_model, H = c->hidden, E = c->n_experts, k = c->top_k;
    if (D % ORC_QK || H % ORC_QK || k < 1 || k > E) return 0;
    uint32_t *idx = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(T ? T : 1) * k);
    float *w = (float *)malloc(sizeof(float) * (size_t)(T ? T : 1) * k);
    float *ybuf = (float *)calloc((size_t)(T ? T : 1) * k * D, sizeof(float));
    float *hbuf = (float *)malloc(sizeof(float) * H);
    float *ysh = (float *)malloc(sizeof(float) * D);
    int ok = idx && w && ybuf && hbuf && ysh;
    for (int t = 0; ok && t < T; t++)
        orc_route_token(c, x + (size_t)t * D, wt->router, idx + (size_t)t * k, w + (size_t)t * k);

    /* Each expert is dequantised once and applied to every token that chose
     * it; per-token results are combined below in the token's sorted order,
     * so the sums match the reference's token-at-a-time loop exactly. */
    for (int e = 0; ok && e < E; e++) {
        int used = 0;
        for (int i = 0; i < T * k && !used; i++) used = (idx[i] == (uint32_t)e && !(w[i] < 1e-6f));
        if (!used) continue;
        expert_f32 m;
        ok = load_expert(c, wt, e, &m);
        for (int i = 0; ok && i < T * k; i++) {
            if (idx[i] != (uint32_t)e || w[i] < 1e-6f) continue; /* model.c:1066 */
            expert_apply(c, &m, x + (size_t)(i / k) * D, ybuf + (size_t)i * D, hbuf);
        }
        free_expert(&m);
    }

    expert_f32 sh = {0, 0, 0};
    int have_sh = wt->gate_shexp && wt->up_shexp && wt->down_shexp;
    if (ok && have_sh) ok = load_expert(c, wt, -1, &sh);
    for (int t = 0; ok && t < T; t++) {
        const float *xt = x + (size_t)t * D;
        float *o = out + (size_t)t * D;
        for (int n = 0; n < D; n++) o[n] = resid ? resid[(size_t)t * D + n] : 0.0f;
        if (have_sh) { /* model.c:1003-1007, optional sigmoid gate */
            expert_apply(c, &sh, xt, ysh, hbuf);
            float gsc = 1.0f;
            if (c->shared_gate && wt->shexp_gate_v) {
                float z = 0.0f;
                for (int d = 0; d < D; d++) z += xt[d] * wt->shexp_gate_v[d];
                gsc = 1.0f / (1.0f + expf(-z));
            }
            for (int n = 0; n < D; n++) o[n] += c->shared_gate ? gsc * ysh[n] : ysh[n];
        }
        /* model.c:1090 then :1142 — routed_out accumulated in sorted order */
        for (int n = 0; n < D; n++) {
            float r = 0.0f;
            for (int a = 0; a < k; a++) {
                size_t i = (size_t)t * k + a;
                if (w[i] < 1e-6f) continue;
                r += w[i] * ybuf[i * D + n];
            }
            o[n] += r;
        }
        if (idx_out) memcpy(idx_out + (size_t)t * k, idx + (size_t)t * k, sizeof(uint32_t) * k);
        if (w_out) memcpy(w_out + (size_t)t * k, w + (size_t)t * k, sizeof(float) * k);
    }
    if (have_sh && sh.g) free_expert(&sh);
    free(idx); free(w); free(ybuf); free(hbuf); free(ysh);
    return ok;
}
