// gpu_backend.cu — the CUDA implementation of ornith-flight's gpu.h API
// (engine/src/gpu.h:29-95), selected at link time in place of gpu.c / the
// Metal backend. Semantics follow the reference backends: synchronous
// compute calls, NULL-safe void calls, size-clamped copies, host-visible
// GPU_BUF_SHARED buffers (CUDA managed memory).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gpu.h"
#include "moe.cuh"
#include "route.cuh"

struct gpu_buffer {
    void *ptr;
    size_t size;
    int flags;
};

struct gpu_context {
    int device;
    cudaStream_t stream;
    size_t used;
    int last_err;
    ofb_workspace *ws;  // cached scratch for gpu_moe_forward / gpu_expert_mlp
    ofb_moe_config ws_cfg;
    int ws_tokens;
    uint32_t *tk_idx;  // device scratch for gpu_topk_softmax
    float *tk_w;
    int tk_cap;
};

namespace {

int fail(gpu_context *ctx, int st) {
    if (ctx && st) ctx->last_err = st;
    return st;
}

int check(gpu_context *ctx, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return OFB_OK;
    return fail(ctx, ofb::cuda_status(e, what));
}

int finish(gpu_context *ctx, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return check(ctx, e, what);
}

int ensure_ws(gpu_context *ctx, const ofb_moe_config *cfg, int tokens) {
    if (ctx->ws && ctx->ws_tokens >= tokens && !memcmp(&ctx->ws_cfg, cfg, sizeof(*cfg))) return OFB_OK;
    if (ctx->ws) {
        cudaStreamSynchronize(ctx->stream);
        ofb_workspace_destroy(ctx->ws);
        ctx->ws = nullptr;
    }
    int want = tokens > ctx->ws_tokens ? tokens : ctx->ws_tokens;
    int st = ofb_workspace_create(cfg, want, &ctx->ws);
    if (st) return fail(ctx, st);
    ctx->ws_cfg = *cfg;
    ctx->ws_tokens = want;
    return OFB_OK;
}

// C[M][N] = A[M][K] B[K][N]; 16x16 tiles, sequential k per output.
__global__ void matmul_f32(float *C, const float *A, const float *B, int M, int N, int K) {
    __shared__ float As[16][17], Bs[16][17];
    const int r = blockIdx.y * 16 + threadIdx.y, c = blockIdx.x * 16 + threadIdx.x;
    float s = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
        As[threadIdx.y][threadIdx.x] = (r < M && ka < K) ? A[(size_t)r * K + ka] : 0.f;
        Bs[threadIdx.y][threadIdx.x] = (kb < K && c < N) ? B[(size_t)kb * N + c] : 0.f;
        __syncthreads();
        for (int kk = 0; kk < 16; kk++) s = __fadd_rn(s, __fmul_rn(As[threadIdx.y][kk], Bs[kk][threadIdx.x]));
        __syncthreads();
    }
    if (r < M && c < N) C[(size_t)r * N + c] = s;
}

// gpu.c:144-156 with the row count honoured: one block per row.
__global__ void rmsnorm_rows(float *out, const float *x, const float *w, int dim) {
    __shared__ float part[32];
    const float *xr = x + (size_t)blockIdx.x * dim;
    float *orow = out + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
    ss = ofb::warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        v = ofb::warp_sum(v);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(part[0] / (float)dim + 1e-6f);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = w[i] * (xr[i] * inv);
}

// gpu.c:158-186 (no clamp in the backend's SiLU)
__global__ void silu_kernel(float *out, const float *x, const float *up, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float v = x[i];
        float s = v / (1.0f + expf(-v));
        out[i] = up ? s * up[i] : s;
    }
}

__global__ void add_kernel(float *out, const float *a, const float *b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

// metal/mlp.metal:49-87 semantics (f32, gate/up [D][H], down [H][D]) in two
// passes: h[j] = silu(x.g_j) * (x.u_j), then out[n] = h . down[:, n].
__global__ void mlp_f32_hidden(float *h, const float *x, const float *g, const float *u, int D, int H) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= H) return;
    float gg = 0.f, uu = 0.f;
    for (int i = 0; i < D; i++) {
        gg += x[i] * g[(size_t)i * H + j];
        uu += x[i] * u[(size_t)i * H + j];
    }
    h[j] = gg / (1.0f + expf(-gg)) * uu;
}

__global__ void mlp_f32_out(float *out, const float *h, const float *dn, int D, int H) {
    int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= D) return;
    float s = 0.f;
    for (int j = 0; j < H; j++) s += h[j] * dn[(size_t)j * D + n];
    out[n] = s;
}

}  // namespace

extern "C" {

gpu_context *gpu_init(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
        ofb::set_error("gpu_init: no CUDA device");
        return nullptr;
    }
    gpu_context *ctx = (gpu_context *)calloc(1, sizeof(gpu_context));
    if (!ctx) return nullptr;
    cudaGetDevice(&ctx->device);
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
        free(ctx);
        return nullptr;
    }
    return ctx;
}

void gpu_destroy(gpu_context *ctx) {
    if (!ctx) return;
    cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) ofb_workspace_destroy(ctx->ws);
    cudaFree(ctx->tk_idx);
    cudaFree(ctx->tk_w);
    cudaStreamDestroy(ctx->stream);
    free(ctx);
}

gpu_buffer *gpu_alloc(gpu_context *ctx, size_t size, gpu_buffer_flags flags) {
    if (!ctx || size == 0) return nullptr;
    gpu_buffer *b = (gpu_buffer *)calloc(1, sizeof(gpu_buffer));
    if (!b) return nullptr;
    cudaError_t e = (flags & GPU_BUF_SHARED) ? cudaMallocManaged(&b->ptr, size) : cudaMalloc(&b->ptr, size);
    if (e == cudaSuccess) e = cudaMemset(b->ptr, 0, size);  // the reference zero-fills (calloc)
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        check(ctx, e, "gpu_alloc");
        if (b->ptr) cudaFree(b->ptr);
        free(b);
        return nullptr;
    }
    b->size = size;
    b->flags = (int)flags;
    ctx->used += size;
    return b;
}

void gpu_free(gpu_context *ctx, gpu_buffer *buf) {
    if (!ctx || !buf) return;
    cudaStreamSynchronize(ctx->stream);
    ctx->used -= buf->size;
    cudaFree(buf->ptr);
    free(buf);
}

void *gpu_get_cpu_ptr(gpu_context *ctx, gpu_buffer *buf) {
    (void)ctx;
    return (buf && (buf->flags & GPU_BUF_SHARED)) ? buf->ptr : nullptr;
}

size_t gpu_buffer_size(gpu_context *ctx, const gpu_buffer *buf) {
    (void)ctx;
    return buf ? buf->size : 0;
}

void gpu_copy_to_device(gpu_context *ctx, gpu_buffer *dst, const void *src, size_t size) {
    if (!ctx || !dst || !src) return;
    size_t n = size < dst->size ? size : dst->size;
    check(ctx, cudaMemcpyAsync(dst->ptr, src, n, cudaMemcpyDefault, ctx->stream), "copy_to_device");
    finish(ctx, "copy_to_device");
}

void gpu_copy_to_host(gpu_context *ctx, void *dst, const gpu_buffer *src, size_t size) {
    if (!ctx || !dst || !src) return;
    size_t n = size < src->size ? size : src->size;
    check(ctx, cudaMemcpyAsync(dst, src->ptr, n, cudaMemcpyDefault, ctx->stream), "copy_to_host");
    finish(ctx, "copy_to_host");
}

void gpu_copy_buffer(gpu_context *ctx, gpu_buffer *dst, const gpu_buffer *src, size_t size) {
    if (!ctx || !dst || !src) return;
    size_t n = size;
    if (n > dst->size) n = dst->size;
    if (n > src->size) n = src->size;
    check(ctx, cudaMemcpyAsync(dst->ptr, src->ptr, n, cudaMemcpyDefault, ctx->stream), "copy_buffer");
    finish(ctx, "copy_buffer");
}

void gpu_matmul(gpu_context *ctx, gpu_buffer *C, const gpu_buffer *A, const gpu_buffer *B, int M,
                int N, int K, quant_mode a_quant, quant_mode b_quant) {
    (void)a_quant;
    if (!ctx || !C || !A || !B || M <= 0 || N <= 0 || K <= 0) return;
    // EXT: B as stored GGUF blocks (Q4_K, Q6_K, F16), element k*N + j: the
    // sequential-sum matvec of dense.cu, bit-identical to dequantise + gpu.c's
    // matmul (gpu.c:104-129)
    int wt = -1;
    size_t bbytes = (size_t)K * N * 4;
    if (b_quant == QUANT_Q4_K) { wt = OFB_TYPE_Q4_K; bbytes = (size_t)K * N / 256 * 144; }
    else if (b_quant == QUANT_Q6_K) { wt = OFB_TYPE_Q6_K; bbytes = (size_t)K * N / 256 * 210; }
    else if (b_quant == QUANT_FP16) { wt = OFB_TYPE_F16; bbytes = (size_t)K * N * 2; }
    if ((size_t)M * N * 4 > C->size || (size_t)M * K * 4 > A->size || bbytes > B->size) {
        ofb::set_error("gpu_matmul: buffer too small for %dx%dx%d", M, N, K);
        fail(ctx, OFB_EINVAL);
        return;
    }
    if (wt >= 0) {
        const int st = ofb_matvec((const float *)A->ptr, M, K, N, B->ptr, wt, (float *)C->ptr, ctx->stream);
        if (st) { fail(ctx, st); return; }
        finish(ctx, "gpu_matmul");
        return;
    }
    dim3 grid((N + 15) / 16, (M + 15) / 16);
    matmul_f32<<<grid, dim3(16, 16), 0, ctx->stream>>>((float *)C->ptr, (const float *)A->ptr,
                                                       (const float *)B->ptr, M, N, K);
    finish(ctx, "gpu_matmul");
}

void gpu_matmul_int4(gpu_context *ctx, gpu_buffer *C, const gpu_buffer *A_quant,
                     const gpu_buffer *A_scale, int M, int N, int K) {
    (void)A_quant;
    (void)A_scale;
    (void)K;
    if (!ctx || !C) return;
    size_t n = (size_t)M * N * 4;
    if (n > C->size) n = C->size;
    check(ctx, cudaMemsetAsync(C->ptr, 0, n, ctx->stream), "gpu_matmul_int4");
    finish(ctx, "gpu_matmul_int4");
}

void gpu_rmsnorm(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x, const gpu_buffer *weight,
                 int rows, int dim) {
    if (!ctx || !out || !x || !weight || dim <= 0) return;
    if (rows < 1) rows = 1;
    rmsnorm_rows<<<rows, 256, 0, ctx->stream>>>((float *)out->ptr, (const float *)x->ptr,
                                                (const float *)weight->ptr, dim);
    finish(ctx, "gpu_rmsnorm");
}

void gpu_silu(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x, int n) {
    if (!ctx || !out || !x || n <= 0) return;
    silu_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>((float *)out->ptr, (const float *)x->ptr, nullptr, n);
    finish(ctx, "gpu_silu");
}

void gpu_silu_mul(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *gate, const gpu_buffer *up, int n) {
    if (!ctx || !out || !gate || !up || n <= 0) return;
    silu_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>((float *)out->ptr, (const float *)gate->ptr,
                                                          (const float *)up->ptr, n);
    finish(ctx, "gpu_silu_mul");
}

void gpu_rope(gpu_context *ctx, gpu_buffer *Q, gpu_buffer *K, int seq_len, int head_dim, int n_heads,
              int n_kv_heads, float base, int pos_start) {
    (void)ctx; (void)Q; (void)K; (void)seq_len; (void)head_dim;
    (void)n_heads; (void)n_kv_heads; (void)base; (void)pos_start;
}

void gpu_attention(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *Q, const gpu_buffer *K_cache,
                   const gpu_buffer *V_cache, int seq_len, int head_dim) {
    (void)ctx; (void)out; (void)Q; (void)K_cache; (void)V_cache; (void)seq_len; (void)head_dim;
}

void gpu_deltanet_step(gpu_context *ctx, gpu_buffer *state, const gpu_buffer *Q, const gpu_buffer *K,
                       const gpu_buffer *V, int dim) {
    (void)ctx; (void)state; (void)Q; (void)K; (void)V; (void)dim;
}

void gpu_expert_mlp(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x, const gpu_buffer *gate_w,
                    const gpu_buffer *up_w, const gpu_buffer *down_w, int d_model, int hidden_dim,
                    quant_mode quant) {
    if (!ctx || !out || !x || !gate_w || !up_w || !down_w || d_model <= 0 || hidden_dim <= 0) return;
    if (quant == QUANT_Q4_K) {
        // one expert, one token: the layer path with a single expert and
        // uniform routing (weight 1/1), no shared expert.
        ofb_moe_config cfg = {d_model, hidden_dim, 1, 1, OFB_LAYOUT_CONTIGUOUS, OFB_ROUTE_FORWARD, 0, 0};
        ofb_moe_weights w = {};
        w.gate_exps = gate_w->ptr;
        w.up_exps = up_w->ptr;
        w.down_exps = down_w->ptr;
        if (ensure_ws(ctx, &cfg, 1)) return;
        int st = ofb_moe_forward(&cfg, &w, (const float *)x->ptr, nullptr, (float *)out->ptr, 1,
                                 nullptr, nullptr, ctx->ws, ctx->stream);
        if (st) { fail(ctx, st); return; }
        finish(ctx, "gpu_expert_mlp");
        return;
    }
    float *h = nullptr;
    if (check(ctx, cudaMallocAsync((void **)&h, (size_t)hidden_dim * 4, ctx->stream), "expert_mlp scratch")) return;
    mlp_f32_hidden<<<(hidden_dim + 127) / 128, 128, 0, ctx->stream>>>(
        h, (const float *)x->ptr, (const float *)gate_w->ptr, (const float *)up_w->ptr, d_model, hidden_dim);
    mlp_f32_out<<<(d_model + 127) / 128, 128, 0, ctx->stream>>>((float *)out->ptr, h,
                                                               (const float *)down_w->ptr, d_model, hidden_dim);
    cudaFreeAsync(h, ctx->stream);
    finish(ctx, "gpu_expert_mlp");
}

void gpu_router(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x, const gpu_buffer *router_weight,
                int d_model, int n_experts) {
    if (!ctx || !out || !x || !router_weight || d_model <= 0 || n_experts <= 0) return;
    int st = ofb::launch_router_logits(OFB_LAYOUT_INTERLEAVED, (const float *)router_weight->ptr,
                                       (const float *)x->ptr, 1, d_model, n_experts, (float *)out->ptr,
                                       ctx->stream);
    if (st) { fail(ctx, st); return; }
    finish(ctx, "gpu_router");
}

void gpu_topk_softmax(gpu_context *ctx, uint32_t *indices, float *weights, const gpu_buffer *logits,
                      int n_experts, int top_k) {
    if (!ctx || !indices || !weights || !logits || n_experts <= 0 || top_k <= 0) return;
    if (n_experts > 1024) n_experts = 1024;  // gpu_metal.m:669 caps at 1024
    if (top_k > n_experts) top_k = n_experts;
    if (top_k > 16) { ofb::set_error("gpu_topk_softmax: top_k > 16"); fail(ctx, OFB_EUNSUPPORTED); return; }
    if (ctx->tk_cap < top_k) {
        cudaFree(ctx->tk_idx);
        cudaFree(ctx->tk_w);
        ctx->tk_idx = nullptr;
        ctx->tk_w = nullptr;
        if (check(ctx, cudaMalloc(&ctx->tk_idx, 16 * 4), "topk scratch") ||
            check(ctx, cudaMalloc(&ctx->tk_w, 16 * 4), "topk scratch"))
            return;
        ctx->tk_cap = 16;
    }
    int st = ofb::launch_route_select((const float *)logits->ptr, 1, n_experts, top_k,
                                      OFB_ROUTE_GET_ROUTING, 0, ctx->tk_idx, ctx->tk_w, ctx->stream);
    if (st) { fail(ctx, st); return; }
    cudaMemcpyAsync(indices, ctx->tk_idx, (size_t)top_k * 4, cudaMemcpyDeviceToHost, ctx->stream);
    cudaMemcpyAsync(weights, ctx->tk_w, (size_t)top_k * 4, cudaMemcpyDeviceToHost, ctx->stream);
    finish(ctx, "gpu_topk_softmax");
}

void gpu_add(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *a, const gpu_buffer *b, int n) {
    if (!ctx || !out || !a || !b || n <= 0) return;
    add_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>((float *)out->ptr, (const float *)a->ptr,
                                                         (const float *)b->ptr, n);
    finish(ctx, "gpu_add");
}

void gpu_sync(gpu_context *ctx) {
    if (!ctx) return;
    check(ctx, cudaStreamSynchronize(ctx->stream), "gpu_sync");
}

size_t gpu_memory_used(gpu_context *ctx) { return ctx ? ctx->used : 0; }

void gpu_print_info(gpu_context *ctx) {
    if (!ctx) return;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, ctx->device) != cudaSuccess) return;
    printf("=== GPU Info (CUDA) ===\n");
    printf("Device:   %s (sm_%d%d, %d SMs)\n", p.name, p.major, p.minor, p.multiProcessorCount);
    printf("HBM:      %.1f GB\n", p.totalGlobalMem / 1e9);
    printf("Memory:   %zu bytes\n", ctx->used);
}

int gpu_last_error(gpu_context *ctx) {
    if (!ctx) return OFB_EINVAL;
    int e = ctx->last_err;
    ctx->last_err = 0;
    return e;
}

void *gpu_get_device_ptr(gpu_context *ctx, gpu_buffer *buf) {
    (void)ctx;
    return buf ? buf->ptr : nullptr;
}

void *gpu_get_stream(gpu_context *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int gpu_moe_forward(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x_norm, const gpu_buffer *resid,
                    const gpu_moe_layer *L, int n_tokens, gpu_buffer *idx_out, gpu_buffer *w_out) {
    if (!ctx) return OFB_EINVAL;
    if (!out || !x_norm || !L || !L->gate_exps || !L->up_exps || !L->down_exps || n_tokens < 0) {
        ofb::set_error("gpu_moe_forward: NULL argument");
        return fail(ctx, OFB_EINVAL);
    }
    ofb_moe_config cfg = {L->d_model, L->hidden, L->n_experts, L->top_k,
                          L->layout, L->routing, L->renorm, L->shared_gate};
    size_t row = (size_t)L->d_model * 4 * n_tokens;
    if (out->size < row || x_norm->size < row || (resid && resid->size < row)) {
        ofb::set_error("gpu_moe_forward: activation buffers smaller than n_tokens x d_model");
        return fail(ctx, OFB_EINVAL);
    }
    int st = ensure_ws(ctx, &cfg, n_tokens > 0 ? n_tokens : 1);
    if (st) return st;
    ofb_moe_weights w;
    w.router = L->router ? (const float *)L->router->ptr : nullptr;
    w.gate_exps = L->gate_exps->ptr;
    w.up_exps = L->up_exps->ptr;
    w.down_exps = L->down_exps->ptr;
    w.gate_shexp = L->gate_shexp ? L->gate_shexp->ptr : nullptr;
    w.up_shexp = L->up_shexp ? L->up_shexp->ptr : nullptr;
    w.down_shexp = L->down_shexp ? L->down_shexp->ptr : nullptr;
    w.shexp_gate = L->shexp_gate ? (const float *)L->shexp_gate->ptr : nullptr;
    st = ofb_moe_forward(&cfg, &w, (const float *)x_norm->ptr, resid ? (const float *)resid->ptr : nullptr,
                         (float *)out->ptr, n_tokens, idx_out ? (uint32_t *)idx_out->ptr : nullptr,
                         w_out ? (float *)w_out->ptr : nullptr, ctx->ws, ctx->stream);
    return fail(ctx, st);
}

}  // extern "C"
