/* forward_main.c — runs the reference's model_load + model_forward for one
 * token of a GGUF file and writes the logits (vocab floats) to a file; built
 * once against the reference's CPU backend (gpu.c) and once against the CUDA
 * backend with the routed experts on gpu_moe_forward, so the two engines can
 * be compared on the same file. usage: forward_main <model.gguf> <token> <out.bin> */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "model.h"
#include "memory.h"

int main(int argc, char **argv) {
    if (argc != 4) { fprintf(stderr, "usage: %s model.gguf token out.bin\n", argv[0]); return 2; }
    memory_config mc;
    memset(&mc, 0, sizeof(mc));
    mc.lru_capacity = 64;
    mc.expert_size_bytes = 4u << 20;
    mc.non_routed_size = 1024;
    char err[256];
    ornith_model *m = model_load(argv[1], &mc, err, sizeof(err), false, false);
    if (!m) { fprintf(stderr, "model_load: %s\n", err); return 1; }
    const model_config *cfg = model_get_config(m);
    const int L = (int)cfg->n_layers, V = (int)cfg->vocab_size;
    const int kv = (int)(cfg->n_kv_heads * cfg->key_length), vv = (int)(cfg->n_kv_heads * cfg->value_length);
    model_buffers b;
    memset(&b, 0, sizeof(b));
    b.max_cache_len = 64;
    b.k_cache = calloc((size_t)L, sizeof(float *));
    b.v_cache = calloc((size_t)L, sizeof(float *));
    b.ssm_conv_states = calloc((size_t)L, sizeof(float *));
    b.ssm_h_states = calloc((size_t)L, sizeof(float *));
    for (int l = 0; l < L; l++) {
        b.k_cache[l] = calloc((size_t)64 * (kv > 0 ? kv : 1), sizeof(float));
        b.v_cache[l] = calloc((size_t)64 * (vv > 0 ? vv : 1), sizeof(float));
        b.ssm_conv_states[l] = calloc((size_t)3 * cfg->d_model * 4, sizeof(float));
        b.ssm_h_states[l] = calloc(4096, sizeof(float));
    }
    float *logits = calloc((size_t)V, sizeof(float));
    model_forward(m, (uint32_t)atoi(argv[2]), logits, &b, 1, 0);
    FILE *f = fopen(argv[3], "wb");
    if (!f || fwrite(logits, sizeof(float), (size_t)V, f) != (size_t)V) { fprintf(stderr, "write failed\n"); return 1; }
    fclose(f);
    model_unload(m);
    return 0;
}
