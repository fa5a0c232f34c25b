/*
 * ornith_moe.h — C ABI of the B200 MoE feed-forward path (raw device pointers).
 *
 * Plain C: pointers, sizes and status codes only. All pointers named "device"
 * are CUDA device (or managed) addresses; `stream` is a cudaStream_t passed as
 * void* (NULL = the legacy default stream). Calls are stream-ordered and do not
 * synchronise unless stated. Every entry point returns OFB_OK (0) or a
 * non-zero OFB_E* status; ofb_last_error() gives a readable reason (per host
 * thread). Nothing here falls back to the CPU.
 *
 * Each entry point names the reference interface it replaces
 * (ornith-flight paths, file:line).
 */
#ifndef ORNITH_MOE_H
#define ORNITH_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    OFB_OK = 0,
    OFB_EINVAL = 1,      /* bad argument (NULL, size, alignment, type) */
    OFB_ECUDA = 2,       /* a CUDA call failed; see ofb_last_error() */
    OFB_ENOMEM = 3,      /* device allocation failed */
    OFB_EUNSUPPORTED = 4,/* shape or mode not supported by this build */
    OFB_ETOOLARGE = 5    /* request exceeds a fixed capacity */
};

/* ggml tensor types (engine/src/third_party/gguf.h:15-22) */
#define OFB_TYPE_F32 0
#define OFB_TYPE_F16 1
#define OFB_TYPE_Q4_K 12
#define OFB_TYPE_Q6_K 14

/* output element types of the dequant entry points */
#define OFB_OUT_F32 0
#define OFB_OUT_BF16 1

/* Expert-tensor layouts.
 * CONTIGUOUS: expert e occupies blocks [e*nb, (e+1)*nb); gate/up rows are
 *   [hidden][d_model] with d_model fastest, down rows [d_model][hidden]; the
 *   router is f32 [n_experts][d_model]. This is the GGUF/llama.cpp layout.
 * INTERLEAVED: the reference's expert-slice semantics
 *   (engine/src/gguf.c:652-711): element i of expert e is linear element
 *   i*n_experts+e; the slices are used as gate/up [d_model][hidden] and down
 *   [hidden][d_model] (engine/src/model.c:351-357, :1085-1088); the router is
 *   f32 [d_model][n_experts] (model.c:1022). Shared-expert tensors follow the
 *   same row convention as the routed ones of the chosen layout. */
#define OFB_LAYOUT_CONTIGUOUS 0
#define OFB_LAYOUT_INTERLEAVED 1

/* Routing variants.
 * FORWARD: model_forward's inline router (engine/src/model.c:1017-1049):
 *   softmax over all experts, exchange-sort the probabilities, keep top_k;
 *   renorm=1 divides the kept probabilities by their sum.
 * GET_ROUTING: model_get_routing (engine/src/model.c:264-321): exchange-sort
 *   the logits, softmax over the kept top_k logits. */
#define OFB_ROUTE_FORWARD 0
#define OFB_ROUTE_GET_ROUTING 1

typedef struct {
    int32_t d_model;     /* multiple of 256 */
    int32_t hidden;      /* expert and shared-expert width, multiple of 256 */
    int32_t n_experts;   /* 1..1024 */
    int32_t top_k;       /* 1..16, <= n_experts */
    int32_t layout;      /* OFB_LAYOUT_* */
    int32_t routing;     /* OFB_ROUTE_* */
    int32_t renorm;      /* 0/1, FORWARD routing only */
    int32_t shared_gate; /* 0/1: scale the shared expert by sigmoid(x . shexp_gate) */
} ofb_moe_config;

/* Device pointers to one layer's weights. gate/up are Q4_K, down is Q6_K.
 * router NULL => uniform routing to experts 0..top_k-1 (model.c:283-289).
 * gate_shexp NULL => no shared expert. */
typedef struct {
    const float *router;
    const void *gate_exps;
    const void *up_exps;
    const void *down_exps;
    const void *gate_shexp;
    const void *up_shexp;
    const void *down_shexp;
    const float *shexp_gate; /* f32 [d_model]; read when shared_gate=1 */
} ofb_moe_weights;

const char *ofb_status_string(int status);
const char *ofb_last_error(void);

/* ---- dequantisation ------------------------------------------------------ */

/* Whole-tensor decode of n_elems elements (multiple of 256 for K-quants) to
 * f32 or bf16 (bf16 = round-to-nearest-even of the bit-exact f32 value).
 * Replaces gguf_dequantize_tensor_from_buf (engine/src/gguf.c:605-638) for
 * Q4_K and Q6_K; f32 output is bit-identical to it. Device pointers. */
int ofb_dequantize(const void *blocks, int type, uint64_t n_elems, void *out, int out_type,
                   void *stream);

/* Expert-slice decode with the expert index fastest-varying: out[i] =
 * element (i*n_experts + expert). Replaces
 * gguf_dequantize_expert_slice_from_buf (engine/src/gguf.c:652-711); same
 * argument checks (expert < 0 or >= n_experts => OFB_EINVAL). */
int ofb_dequantize_expert_slice(const void *blocks, int type, uint64_t n_elems,
                                uint64_t n_experts, int expert, void *out, int out_type,
                                void *stream);

typedef struct ofb_workspace ofb_workspace;

/* ---- routing -------------------------------------------------------------- */

/* Router projection, softmax and top-k for n_tokens rows of x (f32
 * [n_tokens][d_model], device). Writes idx (u32 [n_tokens][top_k]) and w
 * (f32 [n_tokens][top_k]) on the device, bit-identical to the reference's
 * CPU routing (sequential fp32 dot products, the host C library's expf, the
 * exchange sort's tie order). Replaces model_get_routing
 * (engine/src/model.c:264-321) with routing=GET_ROUTING, and gpu_router +
 * gpu_topk_softmax (engine/src/gpu.h:82-87) batched on the device. `ws` is
 * a workspace created for this config with max_tokens >= n_tokens (its logits
 * region is used as scratch). */
int ofb_route(const ofb_moe_config *cfg, const float *router, const float *x, int n_tokens,
              uint32_t *idx, float *w, ofb_workspace *ws, void *stream);

/* The routing ofb_moe_forward uses: top-k indices bit-identical to the
 * reference's, weights within 1e-5 relative of its (an fp32 softmax of logits
 * known to within a rigorous bound of the reference's sequential fp32 sums;
 * tokens whose top-k order the bound cannot certify are recomputed with the
 * reference's exact chain). Contiguous layout with at most 256 experts; other
 * configurations take ofb_route's exact path. Same arguments as ofb_route.
 * Matches model_get_routing / model_forward's router (engine/src/model.c) as
 * stated above. */
int ofb_route_certified(const ofb_moe_config *cfg, const float *router, const float *x, int n_tokens,
                        uint32_t *idx, float *w, ofb_workspace *ws, void *stream);

/* ---- MoE layer --------------------------------------------------------- */

/* Bytes of device scratch one ofb_moe_forward call needs for up to
 * max_tokens tokens. */
size_t ofb_workspace_size(const ofb_moe_config *cfg, int max_tokens);
/* Allocates the scratch (cudaMalloc) on the current device. */
int ofb_workspace_create(const ofb_moe_config *cfg, int max_tokens, ofb_workspace **ws);
int ofb_workspace_destroy(ofb_workspace *ws);

/* One MoE feed-forward layer for n_tokens tokens:
 *   out = resid + g(x) * shared(x) + sum_a w_a * expert_{idx_a}(x)
 * x: f32 [n_tokens][d_model] (the post-norm ffn input, model.c:996);
 * resid: f32 [n_tokens][d_model] or NULL (treated as zero); out may alias
 * resid. idx_out / w_out (optional, device) receive the routing.
 * The routed path and its combine are the block engine/src/model.c:992-1143
 * (refactored out of model_forward); expert SwiGLU = silu(x.G) * (x.U) then
 * . Dn with silu clamped at +-50 (model.c:340-344); experts whose weight is
 * below 1e-6 are skipped (model.c:1066). Stream-ordered, no host sync.
 * Accumulation is fp32 (decode) or bf16 tensor-core with fp32 accumulate
 * (prefill). Routing indices are always bit-exact; weights are bit-exact on
 * the exact path (interleaved layout, no router) and within 1e-5 relative on
 * the certified path (ofb_route_certified, contiguous layout). */
int ofb_moe_forward(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x,
                    const float *resid, float *out, int n_tokens, uint32_t *idx_out,
                    float *w_out, ofb_workspace *ws, void *stream);

/* Same as ofb_moe_forward (routing kept internal), then waits for the layer
 * and reports the device time of its four phases in phase_ms[0..3]:
 * routing (router GEMV + softmax/top-k), dispatch plan, gate/up expert
 * kernel, down + combine. Timing uses CUDA events on `stream`. Diagnostic
 * entry for the benchmark's per-kernel roofline; no reference counterpart. */
int ofb_moe_forward_profiled(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x,
                             const float *resid, float *out, int n_tokens, ofb_workspace *ws,
                             void *stream, float *phase_ms);

/* Counts of tokens routed by ofb_moe_forward's certified decode path since
 * the workspace was created: counts[0] certified directly, counts[1] after
 * recomputing the uncertain candidates exactly, counts[2] after recomputing
 * every logit exactly. Synchronous. Diagnostic; no reference counterpart. */
int ofb_workspace_route_stats(ofb_workspace *ws, int counts[3]);

/* Device-side failures recorded in the workspace since the last call (bit 0:
 * a bulk copy did not complete in time, bit 1: a value another CTA publishes
 * did not arrive in time, bit 2: a tensor-core kernel's pipeline wait
 * expired). Every wait inside this library's kernels is bounded (about half
 * a second); on expiry the kernel records the bit and exits instead of
 * hanging, and its output is not valid. *bits receives the mask, which is
 * then cleared. Synchronous. No reference counterpart. */
int ofb_workspace_device_errors(ofb_workspace *ws, unsigned *bits);

/* ofb_moe_forward without any device allocation, for callers that cannot call
 * cudaMalloc: an engine whose device memory is reserved up front by its own
 * pool or budget (a raw allocation could fail or take memory already
 * promised elsewhere), or a per-token decode loop where allocating would
 * synchronise the device. No counterpart in the reference (its CPU and Metal
 * backends allocate per call).
 * The scratch is one fixed array of ofb_noalloc_capacity() bytes (8 MiB) in
 * device memory, held by every GPU that loads the library until exit; a call
 * whose layer and token count need more returns OFB_ETOOLARGE. The first call
 * on a device looks up the array's device address (make it before any stream
 * capture). All calls share the array: calls whose GPU work overlaps (other
 * streams or host threads) race; calls in one stream are safe. Arguments and
 * results as ofb_moe_forward, without the workspace. */
int ofb_moe_forward_noalloc(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x,
                            const float *resid, float *out, int n_tokens, uint32_t *idx_out,
                            float *w_out, void *stream);
size_t ofb_noalloc_capacity(void);

/* Copies bytes with a kernel (launched with programmatic dependent launch,
 * like the layer kernels), for a decode step's activations between pinned
 * host memory and the device: either pointer may be pinned host memory
 * (device-accessible under unified addressing) or device memory. A few KB
 * this way cost less than a copy-engine transfer and let the next kernel
 * begin its weight loads early. Stream-ordered. No reference counterpart. */
int ofb_copy(void *dst, const void *src, size_t bytes, void *stream);

/* ---- dense projections, LM head and sampling --------------------------------
 * out[t][j] = sum_i x[t][i] * W[i*out_dim + j] for W stored as a GGUF tensor
 * (OFB_TYPE_F32 / F16 / Q4_K / Q6_K, element i*out_dim + j): cpu_matmul_vec
 * over the dequantised weight (engine/src/model.c:351-357, :785-843), and with
 * an F32 [d_model][vocab] weight the LM head (model.c:1219-1231). Every output
 * is a sequential sum with separate multiply and add over the reference's
 * per-element dequant, so results are bit-identical to the reference's. */
int ofb_matvec(const float *x, int n_tokens, int in_dim, int out_dim, const void *w, int w_type, float *out,
               void *stream);
/* model_sample (model.c:1238-1260) for one row of logits on the device:
 * temperature (when > 0 and != 1), softmax with the host library's expf, and
 * the first index whose cumulative probability reaches r in [0, 1) (the
 * caller's uniform draw). scratch: OFB_SAMPLE_SCRATCH(vocab) floats. The sums run in a fixed
 * order (deterministic); the index can differ from the reference's only when
 * r is within ~vocab * 2^-24 of a cumulative boundary. */
#define OFB_SAMPLE_SCRATCH(vocab) ((vocab) + 2 * (((vocab) + 1023) / 1024))
int ofb_sample(const float *logits, int vocab, float temperature, float r, float *scratch, uint32_t *token,
               void *stream);

/* ---- GGUF -> HBM ------------------------------------------------------------
 * Replaces gguf_open / gguf_read_tensor_bytes (engine/src/gguf.c:408-445,
 * 588-601) on the path that feeds the MoE layer: the file is parsed once and a
 * layer's tensors are uploaded as stored (raw Q4_K/Q6_K blocks, F32 router and
 * gate vector), so the experts stay resident in HBM instead of being read
 * per token. Parameters are looked up with the architecture prefix
 * (gguf.c:726-744). layout: OFB_LAYOUT_INTERLEAVED reads the tensors the way
 * the reference's model_forward does (router [d_model][n_experts], expert
 * index fastest, matrices [in][out]); OFB_LAYOUT_CONTIGUOUS reads them in
 * ggml's native order (router rows per expert, each expert's blocks
 * contiguous, matrices [out][in]). Host-side parsing needs no GPU. */
typedef struct ofb_gguf ofb_gguf;
int ofb_gguf_open(const char *path, ofb_gguf **gguf);
int ofb_gguf_close(ofb_gguf *gguf);
/* Type code, dims (fastest first), absolute file offset and byte size (0 when
 * the type's size is unknown) of a tensor. Any output may be NULL. */
int ofb_gguf_tensor(const ofb_gguf *gguf, const char *name, int *type, int *n_dims, uint64_t dims[4],
                    uint64_t *file_offset, uint64_t *n_bytes);
int ofb_gguf_param_u32(const ofb_gguf *gguf, const char *param, uint32_t *value);
/* Copies a tensor's bytes into device memory dst (capacity bytes); synchronous. */
int ofb_gguf_upload(const ofb_gguf *gguf, const char *name, void *dst, uint64_t capacity, void *stream);
typedef struct {
    ofb_moe_config cfg;      /* from the metadata (renorm 1, shared_gate if a gate vector exists) */
    ofb_moe_weights weights; /* device allocations owned by the struct */
} ofb_gguf_moe_layer;
/* blk.<layer>.ffn_{gate,up,down}_exps (required), ffn_gate_inp (router),
 * ffn_{gate,up,down}_shexp and ffn_gate_inp_shexp (optional). */
int ofb_gguf_upload_moe_layer(const ofb_gguf *gguf, int layer, int layout, ofb_gguf_moe_layer *out, void *stream);
int ofb_gguf_free_moe_layer(ofb_gguf_moe_layer *layer);

/* ---- expert parallelism (experts sharded over GPUs) ------------------------
 * Building blocks for one MoE layer whose routed experts are split over
 * n_ranks GPUs, experts_per_rank = n_experts / n_ranks each (rank r owns
 * experts [r*experts_per_rank, (r+1)*experts_per_rank), stored as the
 * CONTIGUOUS layout's expert range); tokens are split too, each rank routing
 * its own. Per layer: ofb_route_certified on own tokens -> ofb_ep_plan + ofb_ep_pack ->
 * all-to-all of rows and metadata (NCCL, by the caller) -> ofb_moe_experts ->
 * all-to-all back -> ofb_moe_shared + ofb_ep_combine. The reference runs its
 * MoE block on one CPU (engine/src/model.c:992-1143) and has no counterpart;
 * the arithmetic per (token, expert) pair is that block's. */
#define OFB_EP_MAX_RANKS 16

/* Dispatch order of a rank's T*K assignments (a = t*K + k, expert idx[a]):
 * grouped by destination rank idx[a] / experts_per_rank, assignment order
 * kept inside a group. Writes send_counts[n_ranks] (int32),
 * slot_of_assignment[T*K] and assignment_of_slot[T*K]. One block; device. */
int ofb_ep_plan(const uint32_t *idx, int n_tokens, int top_k, int experts_per_rank, int n_ranks,
                int32_t *send_counts, int32_t *slot_of_assignment, int32_t *assignment_of_slot,
                void *stream);
/* Send buffers in slot order: send_x[s] = x[token of a] (f32 [d_model]) and
 * send_meta[s] = {expert - dest*experts_per_rank, float bits of w[a]}
 * (int32 pairs), a = assignment_of_slot[s]. */
int ofb_ep_pack(const float *x, const uint32_t *idx, const float *w, int n_tokens, int top_k,
                int d_model, int experts_per_rank, const int32_t *assignment_of_slot, float *send_x,
                int32_t *send_meta, void *stream);
/* out_rows[r] = weight * SwiGLU_e(x_rows[r]) for the row's {local expert e,
 * weight} pair in row_meta (the format ofb_ep_pack writes); routed experts
 * only, cfg->n_experts = experts_per_rank, cfg->top_k = 1, ws created for
 * that cfg with max_tokens >= n_rows. */
int ofb_moe_experts(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x_rows,
                    int n_rows, const int32_t *row_meta, float *out_rows, ofb_workspace *ws,
                    void *stream);
/* out[t] = resid[t] (or 0 when resid is NULL) + g_t * SwiGLU_shared(x[t]),
 * g_t = sigmoid(x[t] . shexp_gate) when cfg->shared_gate and the gate vector
 * is set, else 1. ws: any workspace of this d_model/hidden (contiguous
 * layout) with max_tokens >= n_tokens, e.g. the one ofb_route uses. */
int ofb_moe_shared(const ofb_moe_config *cfg, const ofb_moe_weights *w, const float *x,
                   const float *resid, float *out, int n_tokens, ofb_workspace *ws, void *stream);
/* out[t] += r, r = the sum over k = 0..K-1 (in order) of
 * y_back[slot_of_assignment[t*K+k]] (model.c:1090, :1142 order). */
int ofb_ep_combine(const float *y_back, const int32_t *slot_of_assignment, int n_tokens, int top_k,
                   int d_model, float *out, void *stream);
/* out[t] = x[t] / sqrt(mean(x[t]^2) + eps): the unit-weight RMSNorm that
 * feeds each layer of a layer stack (cpu_rmsnorm, engine/src/model.c:333,
 * with every per-channel weight 1). out may alias x. */
int ofb_rmsnorm(const float *x, int n_tokens, int d_model, float eps, float *out, void *stream);

/* ---- expert parallelism with device-side exchange over NVLink -------------
 * One call per layer, no host synchronisation: rows travel rank to rank as
 * peer stores into a window (device memory every rank of the group maps),
 * with epoch-tagged flags; every wait is bounded (about a second) and
 * records an error instead of hanging (ofb_ep_group_device_errors). Per
 * layer and rank: certified routing of own tokens -> dispatch plan -> rows
 * (bf16 when the receiver's batch takes the tensor-core path, else f32) and
 * {local expert, weight, slot} written into each destination's receive
 * region -> the shared expert on own tokens while rows arrive -> routed
 * experts on the received rows -> each result row stored back into its
 * source's y_back -> the combine in top-k order (model.c:1090, :1142).
 * The reference runs its MoE block on one CPU (engine/src/model.c:992-1143)
 * and has no counterpart; the arithmetic per (token, expert) is that block's.
 *
 * Set-up: ofb_ep_group_create (allocates the window and scratch, returns an
 * IPC handle of OFB_EP_HANDLE_BYTES), the caller gathers every rank's handle
 * (any transport), then ofb_ep_group_connect opens the peers' windows;
 * ofb_ep_group_create_nccl does both with an ncclComm_t (libnccl loaded at
 * run time). Every rank must call ofb_ep_layer_forward for the same layers
 * in the same order (the epochs advance together). */
#define OFB_EP_HANDLE_BYTES 64
typedef struct ofb_ep_group ofb_ep_group;
int ofb_ep_group_create(const ofb_moe_config *cfg, int rank, int n_ranks, int max_tokens_per_rank,
                        ofb_ep_group **group, void *ipc_handle_out);
int ofb_ep_group_connect(ofb_ep_group *group, const void *all_handles /* n_ranks * OFB_EP_HANDLE_BYTES */);
int ofb_ep_group_create_nccl(const ofb_moe_config *cfg, void *nccl_comm, int max_tokens_per_rank,
                             ofb_ep_group **group, void *stream);
int ofb_ep_group_destroy(ofb_ep_group *group);
/* w: the full router, the shared expert and gate vector, and this rank's
 * routed experts [rank*E/n, (rank+1)*E/n) (contiguous layout, 16-byte
 * aligned). out = resid + g*shared(x) + sum_k w_k expert_k(x) for this rank's
 * n_tokens tokens x; out may alias resid but not x. */
int ofb_ep_layer_forward(ofb_ep_group *group, const ofb_moe_weights *w, const float *x, const float *resid,
                         float *out, int n_tokens, void *stream);
/* Bits of expired device waits since the last call (bit 0: rows or flags of
 * a peer did not arrive in time); cleared by the call. Synchronous. */
int ofb_ep_group_device_errors(ofb_ep_group *group, unsigned *bits);

/* ---- seeded synthetic inputs ---------------------------------------------- */

/* Fills n_blocks Q4_K or Q6_K super-blocks on the device from a counter-based
 * generator (SplitMix64 finaliser over (seed, stream_id, word index)): every
 * quant and scale byte uniform; d and dmin = fp16(round-to-nearest-even of
 * U(0, 0.01)). ofb_synth_blocks_host produces the same bytes on the host. */
int ofb_synth_blocks(void *dst, int type, uint64_t n_blocks, uint64_t first_block,
                     uint64_t seed, uint64_t stream_id, void *stream);
void ofb_synth_blocks_host(void *dst, int type, uint64_t n_blocks, uint64_t first_block,
                           uint64_t seed, uint64_t stream_id);
/* n host floats drawn N(0, sigma^2) (Box-Muller over the same generator). */
void ofb_synth_normal_host(float *dst, uint64_t n, uint64_t seed, uint64_t stream_id,
                           float sigma);

/* Library build identification (sm_100a kernels). */
const char *ofb_build_info(void);

#ifdef __cplusplus
}
#endif
#endif
