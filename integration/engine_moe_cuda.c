/* engine_moe_cuda.c — engine-side glue (C99) that runs model_forward's routed
 * experts (engine/src/model.c:1011-1138) through the CUDA backend's
 * gpu_moe_forward. On a layer's first use the router and the three fused
 * expert tensors are uploaded to device buffers as stored in the GGUF file
 * (raw Q4_K / Q6_K blocks, read with gguf_read_tensor_data) and kept for the
 * life of the process: every expert is resident, no per-token slice decode.
 * The tensors are read the way the reference reads them (router [D][E],
 * expert index fastest: OFB_LAYOUT_INTERLEAVED) with the reference's routing
 * (softmax over all experts, top-k, no renormalisation, no shared-expert gate;
 * the shared expert stays in model_forward's own code). */
#include "engine_moe_cuda.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define OFB_LAYOUT_INTERLEAVED 1
#define OFB_ROUTE_FORWARD 0
#define MAX_LAYERS 256

typedef struct {
    gpu_buffer *router, *gate, *up, *down;
} layer_bufs;
static layer_bufs g_layers[MAX_LAYERS];

static gpu_buffer *upload_tensor(gpu_context *gpu, const gguf_model *gguf, int layer, const char *what) {
    char name[128];
    snprintf(name, sizeof(name), "blk.%d.%s", layer, what);
    const gguf_tensor_info *t = gguf_find_tensor(gguf, name);
    if (!t) return NULL;
    void *host = malloc(t->size_bytes);
    gpu_buffer *b = host ? gpu_alloc(gpu, t->size_bytes, 0) : NULL;
    if (b && gguf_read_tensor_data(gguf, t, host, t->size_bytes) == t->size_bytes)
        gpu_copy_to_device(gpu, b, host, t->size_bytes);
    free(host);
    return b;
}

void ofb_engine_moe_routed(gpu_context *gpu, const gguf_model *gguf, const model_config *cfg, int layer,
                           const float *router_f32, const float *ffn_x, float *routed_out) {
    const int D = (int)cfg->d_model, E = (int)cfg->n_experts_per_layer;
    memset(routed_out, 0, (size_t)D * sizeof(float));
    if (layer < 0 || layer >= MAX_LAYERS) return;
    layer_bufs *L = &g_layers[layer];
    if (!L->router) {
        L->router = gpu_alloc(gpu, (size_t)D * E * sizeof(float), 0);
        if (L->router) gpu_copy_to_device(gpu, L->router, router_f32, (size_t)D * E * sizeof(float));
        L->gate = upload_tensor(gpu, gguf, layer, "ffn_gate_exps.weight");
        L->up = upload_tensor(gpu, gguf, layer, "ffn_up_exps.weight");
        L->down = upload_tensor(gpu, gguf, layer, "ffn_down_exps.weight");
    }
    if (!L->router || !L->gate || !L->up || !L->down) return;
    gpu_moe_layer ml;
    memset(&ml, 0, sizeof(ml));
    ml.d_model = D;
    ml.hidden = (int32_t)cfg->expert_hidden_dim;
    ml.n_experts = E;
    ml.top_k = (int32_t)cfg->n_active_experts;
    ml.layout = OFB_LAYOUT_INTERLEAVED;
    ml.routing = OFB_ROUTE_FORWARD;
    ml.renorm = 0;
    ml.shared_gate = 0;
    ml.router = L->router;
    ml.gate_exps = L->gate;
    ml.up_exps = L->up;
    ml.down_exps = L->down;
    gpu_buffer *xb = gpu_alloc(gpu, (size_t)D * sizeof(float), 0);
    gpu_buffer *ob = gpu_alloc(gpu, (size_t)D * sizeof(float), 0);
    if (xb && ob) {
        gpu_copy_to_device(gpu, xb, ffn_x, (size_t)D * sizeof(float));
        if (gpu_moe_forward(gpu, ob, xb, NULL, &ml, 1, NULL, NULL) == 0) {
            gpu_sync(gpu);
            gpu_copy_to_host(gpu, routed_out, ob, (size_t)D * sizeof(float));
        } else {
            fprintf(stderr, "gpu_moe_forward failed (layer %d)\n", layer);
        }
    }
    gpu_free(gpu, xb);
    gpu_free(gpu, ob);
}
