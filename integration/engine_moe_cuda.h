/* engine_moe_cuda.h — the routed-expert block of model_forward on the CUDA
 * backend (see engine_moe_cuda.c). */
#ifndef ENGINE_MOE_CUDA_H
#define ENGINE_MOE_CUDA_H
#include "gguf.h"
#include "gpu.h"
#include "model.h"

/* routed_out[D] = sum over the top-k experts of w * SwiGLU_e(ffn_x), the
 * reference's routing (softmax over all experts, top-k, no renormalisation,
 * skip below 1e-6), expert weights read from the GGUF file as stored. */
void ofb_engine_moe_routed(gpu_context *gpu, const gguf_model *gguf, const model_config *cfg, int layer,
                           const float *router_f32, const float *ffn_x, float *routed_out);
#endif
