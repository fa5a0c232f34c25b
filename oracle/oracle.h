/*
 * oracle.h — CPU restatement of ornith-flight's MoE feed-forward arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; it is linked by tests/, by __graft_entry__.smoke() and by
 * bench.py's cpu_baseline / reference legs, never by the product library.
 *
 * Every function restates the reference's C99 code in plain C with the same
 * operation order (sequential fp32 sums, separate multiply and add, glibc
 * expf) and cites the reference file:line it follows (paths are relative to
 * the ornith-flight project root). Build flags: -O2 -ffp-contract=off on the
 * x86-64 baseline ISA (no FMA), the flags the reference's CPU path is
 * measured with.
 *
 * Parity pinning: the dequant functions are checked bit-for-bit against the
 * reference's own engine/src/gguf.c compiled unmodified into oracle/_ref/
 * (tests/golden/ holds fixtures generated from it). The routing/MoE block is
 * a restatement of engine/src/model.c:992-1143 (inline in model_forward, not
 * callable on its own); its renormalise and shared-gate options are defined
 * by the task, not by reference code (model.c has neither).
 */
#ifndef ORNITH_ORACLE_H
#define ORNITH_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 256
#define ORC_Q4K_BYTES 144
#define ORC_Q6K_BYTES 210

/* ggml type codes, engine/src/third_party/gguf.h:15-22 */
#define ORC_TYPE_F32 0
#define ORC_TYPE_F16 1
#define ORC_TYPE_Q4_K 12
#define ORC_TYPE_Q6_K 14

float orc_fp16_to_fp32(uint16_t h);
void orc_q4k_block(const uint8_t *blk, float *y);
void orc_q6k_block(const uint8_t *blk, float *y);
float orc_q4k_one(const uint8_t *blk, int pos);
float orc_q6k_one(const uint8_t *blk, int pos);
/* whole-tensor decode; returns 1 on success, 0 on unsupported type / NULL */
int orc_dequant_tensor(const void *data, int type, uint64_t n_elems, float *out);
/* expert slice, expert index fastest-varying (interleaved layout) */
int orc_dequant_slice(const void *data, int type, uint64_t n_elems,
                      uint64_t n_experts, int expert, float *out);

typedef int (*orc_tensor_fn)(const void *, int, uint64_t, float *);
typedef int (*orc_slice_fn)(const void *, int, uint64_t, uint64_t, int, float *);
/* Route the layer's dequant through other implementations (NULL = restatement). */
void orc_set_dequant(orc_tensor_fn t, orc_slice_fn s);

/* MoE layer ------------------------------------------------------------- */
#define ORC_LAYOUT_CONTIGUOUS 0   /* expert e = contiguous blocks, rows K-fastest */
#define ORC_LAYOUT_INTERLEAVED 1  /* the reference's expert-fastest slices */

#define ORC_ROUTE_FORWARD 0       /* model_forward: softmax(all), sort probs */
#define ORC_ROUTE_GET_ROUTING 1   /* model_get_routing: sort logits, softmax(top-k) */

typedef struct {
    int d_model, hidden, n_experts, top_k;
    int layout;       /* ORC_LAYOUT_* */
    int routing;      /* ORC_ROUTE_* */
    int renorm;       /* ORC_ROUTE_FORWARD only: divide top-k probs by their sum */
    int shared_gate;  /* multiply the shared expert by sigmoid(x . v) */
} orc_moe_cfg;

typedef struct {
    const float *router;     /* contiguous: [E][D]; interleaved: [D][E]; NULL => uniform */
    const void *gate_exps;   /* Q4_K */
    const void *up_exps;     /* Q4_K */
    const void *down_exps;   /* Q6_K */
    const void *gate_shexp;  /* Q4_K, NULL => no shared expert */
    const void *up_shexp;    /* Q4_K */
    const void *down_shexp;  /* Q6_K */
    const float *shexp_gate_v; /* [D], used when shared_gate */
} orc_moe_weights;

float orc_expf(float x);
void orc_expf_batch(const float *x, float *out, uint64_t n);
float orc_silu(float x);
void orc_route_token(const orc_moe_cfg *cfg, const float *x, const float *router,
                     uint32_t *idx, float *w);
/* out[T][D] = resid + shared(x) + sum_a w_a * expert_a(x); resid may be NULL.
 * idx/w (T x top_k) receive the routing; either may be NULL. Returns 0 on bad args. */
int orc_moe_forward(const orc_moe_cfg *cfg, const orc_moe_weights *wt,
                    const float *x, const float *resid, int n_tokens, float *out,
                    uint32_t *idx, float *w);

/* seeded synthetic inputs: the same bytes / floats as the library's
 * ofb_synth_blocks_host / ofb_synth_normal_host (synth.c) */
void orc_synth_blocks(void *dst, int type, uint64_t n_blocks, uint64_t first_block, uint64_t seed,
                      uint64_t stream_id);
void orc_synth_normal(float *dst, uint64_t n, uint64_t seed, uint64_t stream_id, float sigma);

/* reference CPU matmul semantics used by the gpu.h contract (gpu.c:104-115) */
void orc_matmul(float *C, const float *A, const float *B, int M, int N, int K);

#ifdef __cplusplus
}
#endif
#endif
