/*
 * gpu.h — ornith-flight's GPU-abstraction API, implemented by the CUDA
 * backend (libornith_cuda.so). The declarations keep the reference's names,
 * argument order and meaning (engine/src/gpu.h:12-95) so that engine/src
 * links against this backend in place of gpu.c (CPU) or gpu_metal.m (Metal),
 * exactly as the reference swaps those two (engine/Makefile:75-84,113-131).
 *
 * Semantics kept from the reference backends:
 *  - gpu_alloc returns NULL for size 0 or on failure (gpu.c:40-56);
 *    GPU_BUF_SHARED buffers are host-dereferenceable via gpu_get_cpu_ptr
 *    (t_gpu.c:46-66): CUDA managed memory here. Default buffers are device
 *    memory; gpu_get_cpu_ptr returns NULL for them.
 *  - copies clamp to the buffer size (gpu.c:76-102).
 *  - every compute call is complete when it returns (Metal commits and
 *    waits, gpu_metal.m:359-360); void calls return silently on NULL
 *    arguments (gpu.c:123). The CUDA backend records the failure reason,
 *    readable with gpu_last_error().
 *
 * Additive, ABI-compatible extensions (marked EXT): K-quant members of
 * quant_mode, gpu_last_error, device-pointer/stream access, and the batched
 * gpu_moe_forward layer entry.
 */
#ifndef ORNITH_GPU_H
#define ORNITH_GPU_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gpu_context gpu_context;
typedef struct gpu_buffer gpu_buffer;

/* engine/src/gpu.h:15-20, plus EXT members appended (values unchanged). */
typedef enum {
    QUANT_NONE = 0,
    QUANT_FP16,
    QUANT_INT8,
    QUANT_INT4,
    QUANT_Q4_K, /* EXT: gate/up Q4_K super-blocks, down Q6_K (the GGUF expert mix) */
    QUANT_Q6_K, /* EXT: Q6_K super-blocks */
} quant_mode;

/* engine/src/gpu.h:22-26 */
typedef enum {
    GPU_BUF_DEFAULT = 0,
    GPU_BUF_SHARED = 1 << 0,
    GPU_BUF_CONSTANT = 1 << 1,
} gpu_buffer_flags;

/* Lifecycle — engine/src/gpu.h:29-30 */
gpu_context *gpu_init(void);
void gpu_destroy(gpu_context *ctx);

/* Buffers — engine/src/gpu.h:33-43 */
gpu_buffer *gpu_alloc(gpu_context *ctx, size_t size, gpu_buffer_flags flags);
void gpu_free(gpu_context *ctx, gpu_buffer *buf);
void *gpu_get_cpu_ptr(gpu_context *ctx, gpu_buffer *buf);
size_t gpu_buffer_size(gpu_context *ctx, const gpu_buffer *buf);
void gpu_copy_to_device(gpu_context *ctx, gpu_buffer *dst, const void *src, size_t size);
void gpu_copy_to_host(gpu_context *ctx, void *dst, const gpu_buffer *src, size_t size);
void gpu_copy_buffer(gpu_context *ctx, gpu_buffer *dst, const gpu_buffer *src, size_t size);

/* Compute — engine/src/gpu.h:46-90 */
/* C[M][N] = A[M][K] . B[K][N], row-major f32 (gpu.c:104-129). */
void gpu_matmul(gpu_context *ctx, gpu_buffer *C, const gpu_buffer *A, const gpu_buffer *B,
                int M, int N, int K, quant_mode a_quant, quant_mode b_quant);
/* The reference's CPU backend zero-fills C (gpu.c:131-140); kept. */
void gpu_matmul_int4(gpu_context *ctx, gpu_buffer *C, const gpu_buffer *A_quant,
                     const gpu_buffer *A_scale, int M, int N, int K);
void gpu_rmsnorm(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x,
                 const gpu_buffer *weight, int rows, int dim);
void gpu_silu(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x, int n);
void gpu_silu_mul(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *gate,
                  const gpu_buffer *up, int n);
/* Not on the MoE path; no-ops as in the reference's CPU backend (gpu.c:188-206). */
void gpu_rope(gpu_context *ctx, gpu_buffer *Q, gpu_buffer *K, int seq_len, int head_dim,
              int n_heads, int n_kv_heads, float base, int pos_start);
void gpu_attention(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *Q,
                   const gpu_buffer *K_cache, const gpu_buffer *V_cache, int seq_len,
                   int head_dim);
void gpu_deltanet_step(gpu_context *ctx, gpu_buffer *state, const gpu_buffer *Q,
                       const gpu_buffer *K, const gpu_buffer *V, int dim);
/* One expert SwiGLU for one token. quant == QUANT_NONE: f32 weights with the
 * Metal kernel's layout gate/up [d_model][hidden], down [hidden][d_model]
 * (metal/mlp.metal:40-87). quant == QUANT_Q4_K (EXT): gate/up Q4_K rows
 * [hidden][d_model], down Q6_K rows [d_model][hidden] (contiguous layout). */
void gpu_expert_mlp(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x,
                    const gpu_buffer *gate_w, const gpu_buffer *up_w,
                    const gpu_buffer *down_w, int d_model, int hidden_dim, quant_mode quant);
/* logits[E] = x[D] . W[D][E] (metal/mlp.metal:94-109), sequential fp32. */
void gpu_router(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x,
                const gpu_buffer *router_weight, int d_model, int n_experts);
/* Top-k of device logits, softmax over the kept logits; indices/weights are
 * HOST pointers (gpu_metal.m:663-685). */
void gpu_topk_softmax(gpu_context *ctx, uint32_t *indices, float *weights,
                      const gpu_buffer *logits, int n_experts, int top_k);
void gpu_add(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *a, const gpu_buffer *b, int n);

/* Sync / info — engine/src/gpu.h:93-95 */
void gpu_sync(gpu_context *ctx);
size_t gpu_memory_used(gpu_context *ctx);
void gpu_print_info(gpu_context *ctx);

/* ---- EXT -------------------------------------------------------------- */

/* Status of the last failed call on this context (0 = none); cleared by
 * reading. Values are the OFB_* codes of ornith_moe.h. */
int gpu_last_error(gpu_context *ctx);
/* Device address of a buffer, for passing to the ofb_* entry points. */
void *gpu_get_device_ptr(gpu_context *ctx, gpu_buffer *buf);
/* The context's CUDA stream (cudaStream_t as void*). */
void *gpu_get_stream(gpu_context *ctx);

/* One layer's MoE weights as backend buffers (see ornith_moe.h for the
 * meaning of every field). */
typedef struct {
    int32_t d_model, hidden, n_experts, top_k;
    int32_t layout;      /* OFB_LAYOUT_* */
    int32_t routing;     /* OFB_ROUTE_* */
    int32_t renorm;
    int32_t shared_gate;
    const gpu_buffer *router;
    const gpu_buffer *gate_exps, *up_exps, *down_exps;
    const gpu_buffer *gate_shexp, *up_shexp, *down_shexp; /* NULL => no shared expert */
    const gpu_buffer *shexp_gate;
} gpu_moe_layer;

/* The MoE block of engine/src/model.c:992-1143 for n_tokens rows at once:
 * out = resid + shared + routed (resid may be NULL). Stream-ordered on the
 * context's stream: call gpu_sync() before reading results on the host.
 * idx_out / w_out are optional device buffers (u32 / f32, n_tokens*top_k).
 * Returns an OFB_* status. */
int gpu_moe_forward(gpu_context *ctx, gpu_buffer *out, const gpu_buffer *x_norm,
                    const gpu_buffer *resid, const gpu_moe_layer *layer, int n_tokens,
                    gpu_buffer *idx_out, gpu_buffer *w_out);

#ifdef __cplusplus
}
#endif
#endif
