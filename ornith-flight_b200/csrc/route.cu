// route.cu — bit-exact routing on the device.
//
// The reference routes on the CPU (engine/src/model.c:1017-1049 inline in
// model_forward; model.c:264-321 model_get_routing):
//   logit[e] = sequential fp32 sum over d of x[d]*W(e,d), separate mul/add;
//   softmax = max, expf(l - max), sequential sum over e, divide;
//   selection = exchange sort (strict '>' swaps) of the first k positions.
// Every one of these steps is reproduced exactly:
//   * logits: one thread owns one (token, expert) chain and walks d in order
//     with __fmul_rn/__fadd_rn. Decode (few tokens) streams each router row
//     straight from global memory; prefill tiles 64 tokens x 64 experts
//     through shared memory so the router is read once per tile.
//   * expf: ofb_exact_expf (exact_expf.h) reproduces the host C library.
//   * the exchange sort is emulated pass by pass with a warp scan (see
//     exchange_pass), so ties resolve exactly as the reference's swaps do.
#include <cfloat>

#include "common.cuh"
#include "exact_expf.h"
#include "route.cuh"
#include "exchange.cuh"

namespace ofb {

// ---- router logits, few tokens: one thread per (token, expert) -----------
// grid (ceil(E/128), T), block 128; x[t] staged in shared memory.
template <int LAYOUT>
__global__ void __launch_bounds__(128) router_logits_rows(const float *__restrict__ W,
                                                          const float *__restrict__ x, int D, int E,
                                                          float *__restrict__ logits) {
    extern __shared__ float xs[];
    const int t = blockIdx.y;
    const float *xt = x + (size_t)t * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) xs[i] = xt[i];
    __syncthreads();
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    float s = 0.0f;
    if (LAYOUT == OFB_LAYOUT_CONTIGUOUS) {
        const float4 *row = reinterpret_cast<const float4 *>(W + (size_t)e * D);
#pragma unroll 8
        for (int d4 = 0; d4 < D / 4; d4++) {
            float4 w = __ldg(row + d4);
            s = __fadd_rn(s, __fmul_rn(xs[4 * d4 + 0], w.x));
            s = __fadd_rn(s, __fmul_rn(xs[4 * d4 + 1], w.y));
            s = __fadd_rn(s, __fmul_rn(xs[4 * d4 + 2], w.z));
            s = __fadd_rn(s, __fmul_rn(xs[4 * d4 + 3], w.w));
        }
    } else {
#pragma unroll 8
        for (int d = 0; d < D; d++) s = __fadd_rn(s, __fmul_rn(xs[d], __ldg(W + (size_t)d * E + e)));
    }
    logits[(size_t)t * E + e] = s;
}

// ---- router logits, many tokens: 64x64 tile, 4x4 chains per thread -------
constexpr int RT_T = 64, RT_E = 64, RT_D = 32;
template <int LAYOUT>
__global__ void __launch_bounds__(256) router_logits_tiled(const float *__restrict__ W,
                                                           const float *__restrict__ x, int T, int D,
                                                           int E, float *__restrict__ logits) {
    __shared__ __align__(16) float Xs[2][RT_D][RT_T];
    __shared__ __align__(16) float Ws[2][RT_D][RT_E];
    const int t0 = blockIdx.y * RT_T, e0 = blockIdx.x * RT_E;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    auto load = [&](int buf, int d0) {
        // 64 rows x 32 d of x and of W: 2048 floats each, 8 per thread.
        for (int i = tid; i < RT_T * RT_D; i += 256) {
            int r = i / RT_D, dd = i % RT_D;
            int t = t0 + r;
            Xs[buf][dd][r] = (t < T) ? x[(size_t)t * D + d0 + dd] : 0.0f;
        }
        if (LAYOUT == OFB_LAYOUT_CONTIGUOUS) {
            for (int i = tid; i < RT_E * RT_D; i += 256) {
                int r = i / RT_D, dd = i % RT_D;
                int e = e0 + r;
                Ws[buf][dd][r] = (e < E) ? __ldg(W + (size_t)e * D + d0 + dd) : 0.0f;
            }
        } else {
            for (int i = tid; i < RT_E * RT_D; i += 256) {
                int dd = i / RT_E, r = i % RT_E;
                int e = e0 + r;
                Ws[buf][dd][r] = (e < E) ? __ldg(W + (size_t)(d0 + dd) * E + e) : 0.0f;
            }
        }
    };

    load(0, 0);
    __syncthreads();
    const int nchunks = D / RT_D;
    for (int c = 0; c < nchunks; c++) {
        const int buf = c & 1;
        if (c + 1 < nchunks) load(buf ^ 1, (c + 1) * RT_D);
#pragma unroll 4
        for (int dd = 0; dd < RT_D; dd++) {
            float4 xv = *reinterpret_cast<const float4 *>(&Xs[buf][dd][ty * 4]);
            float4 wv = *reinterpret_cast<const float4 *>(&Ws[buf][dd][tx * 4]);
            float xa[4] = {xv.x, xv.y, xv.z, xv.w};
            float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xa[i], wa[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int t = t0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int e = e0 + tx * 4 + j;
            if (e < E) logits[(size_t)t * E + e] = acc[i][j];
        }
    }
}

// ---- softmax + top-k, one warp per token ---------------------------------
// Shared memory per warp: 4*E floats/ints.
__global__ void __launch_bounds__(128) route_select(const float *__restrict__ logits, int T, int E,
                                                    int K, int routing, int renorm,
                                                    uint32_t *__restrict__ idx_out,
                                                    float *__restrict__ w_out) {
    extern __shared__ float sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int t = blockIdx.x * (blockDim.x >> 5) + wib;
    if (t >= T) return;
    float *val = sm + (size_t)wib * 4 * E;
    int *id = reinterpret_cast<int *>(val + E);
    float *oval = val + 2 * E;
    int *oid = reinterpret_cast<int *>(val + 3 * E);
    const float *lg = logits + (size_t)t * E;
    for (int e = lane; e < E; e += 32) { val[e] = lg[e]; id[e] = e; }
    __syncwarp();
    if (routing == OFB_ROUTE_GET_ROUTING) {
        exchange_topk(val, id, oval, oid, E, K, lane);
        if (lane == 0) {
            // model.c:306-317: softmax over the kept logits
            float mx = val[0], sum = 0.0f, s[16];
            for (int a = 0; a < K; a++) { s[a] = ofb_exact_expf(__fsub_rn(val[a], mx)); sum = __fadd_rn(sum, s[a]); }
            for (int a = 0; a < K; a++) {
                w_out[(size_t)t * K + a] = __fdiv_rn(s[a], sum);
                idx_out[(size_t)t * K + a] = (uint32_t)id[a];
            }
        }
        return;
    }
    // model.c:1027-1035: max (sequential strict '>' => the maximum value),
    // exp, sequential sum, divide.
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, val[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) val[e] = ofb_exact_expf(__fsub_rn(val[e], mx));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, val[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) val[e] = __fdiv_rn(val[e], sum);
    __syncwarp();
    exchange_topk(val, id, oval, oid, E, K, lane);
    if (lane == 0) {
        float ssum = 0.0f;
        for (int a = 0; a < K; a++) ssum = __fadd_rn(ssum, val[a]);
        for (int a = 0; a < K; a++) {
            idx_out[(size_t)t * K + a] = (uint32_t)id[a];
            w_out[(size_t)t * K + a] = renorm ? __fdiv_rn(val[a], ssum) : val[a];
        }
    }
}

// model.c:283-289: no router tensor => experts 0..k-1 with weight 1/k.
__global__ void route_uniform(int T, int K, uint32_t *idx_out, float *w_out) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < T * K) {
        idx_out[i] = (uint32_t)(i % K);
        w_out[i] = __fdiv_rn(1.0f, (float)K);
    }
}

int launch_router_logits(int layout, const float *W, const float *x, int T, int D, int E,
                         float *logits, cudaStream_t s) {
    if (T <= 0) return OFB_OK;
    if (T < 16) {
        dim3 grid((E + 127) / 128, T);
        size_t smem = (size_t)D * sizeof(float);
        if (smem > 48 * 1024) {
            auto k = (layout == OFB_LAYOUT_CONTIGUOUS) ? router_logits_rows<OFB_LAYOUT_CONTIGUOUS>
                                                       : router_logits_rows<OFB_LAYOUT_INTERLEAVED>;
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        }
        if (layout == OFB_LAYOUT_CONTIGUOUS)
            router_logits_rows<OFB_LAYOUT_CONTIGUOUS><<<grid, 128, smem, s>>>(W, x, D, E, logits);
        else
            router_logits_rows<OFB_LAYOUT_INTERLEAVED><<<grid, 128, smem, s>>>(W, x, D, E, logits);
    } else {
        dim3 grid((E + RT_E - 1) / RT_E, (T + RT_T - 1) / RT_T);
        if (layout == OFB_LAYOUT_CONTIGUOUS)
            router_logits_tiled<OFB_LAYOUT_CONTIGUOUS><<<grid, 256, 0, s>>>(W, x, T, D, E, logits);
        else
            router_logits_tiled<OFB_LAYOUT_INTERLEAVED><<<grid, 256, 0, s>>>(W, x, T, D, E, logits);
    }
    OFB_CHECK_LAUNCH("router logits");
    return OFB_OK;
}

int launch_route_select(const float *logits, int T, int E, int K, int routing, int renorm,
                        uint32_t *idx, float *w, cudaStream_t s) {
    if (T <= 0) return OFB_OK;
    const int warps = 4;
    size_t smem = (size_t)warps * 4 * E * sizeof(float);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(route_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    route_select<<<(T + warps - 1) / warps, warps * 32, smem, s>>>(logits, T, E, K, routing, renorm, idx, w);
    OFB_CHECK_LAUNCH("route select");
    return OFB_OK;
}

int launch_route_uniform(int T, int K, uint32_t *idx, float *w, cudaStream_t s) {
    if (T <= 0) return OFB_OK;
    route_uniform<<<(T * K + 255) / 256, 256, 0, s>>>(T, K, idx, w);
    OFB_CHECK_LAUNCH("route uniform");
    return OFB_OK;
}

}  // namespace ofb
