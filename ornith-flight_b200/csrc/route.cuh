// route.cuh — internal launchers shared by the routing, MoE and gpu.h layers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ofb {

// logits[T][E] from x[T][D] and the router (layout per OFB_LAYOUT_*),
// sequential fp32 per (token, expert).
int launch_router_logits(int layout, const float *W, const float *x, int T, int D, int E,
                         float *logits, cudaStream_t s);
// softmax / exchange-sort selection of logits[T][E] -> idx[T][K], w[T][K].
int launch_route_select(const float *logits, int T, int E, int K, int routing, int renorm,
                        uint32_t *idx, float *w, cudaStream_t s);
int launch_route_uniform(int T, int K, uint32_t *idx, float *w, cudaStream_t s);

}  // namespace ofb
