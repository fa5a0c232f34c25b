// dense.cu — the non-MoE matrix-vector products of the forward pass on the
// raw tensors, and sampling.
//
// ofb_matvec: out[t][j] = sum_i x[t][i] * W[i*out_dim + j] with W stored as a
// GGUF tensor (F32, F16, Q4_K or Q6_K; element i*out_dim + j, blocks along
// the output index). This is cpu_matmul_vec over a fully dequantised weight
// (engine/src/model.c:351-357 after load_tensor, :785-843): the attention /
// SSM projections, and with an F32 [d_model][vocab] weight the LM head
// (model.c:1219-1231). Each output is one thread's sequential sum over i with
// a separate multiply and add, every weight decoded with the reference's
// per-element arithmetic, so the results are bit-identical to the reference's
// dequantise-then-multiply. HBM-bound: consecutive threads read consecutive
// weights of one input row (coalesced), each weight once per group of up to
// MV_T tokens; x lives in shared memory.
//
// ofb_sample: model_sample (model.c:1238-1260) on device for one row of
// logits: divide by the temperature (when > 0 and != 1), softmax with the
// host library's expf, and the first index whose cumulative probability
// reaches r. The reference sums the 248k probabilities sequentially; here the
// sums are fixed-order trees and scans over 1024-logit chunks spread over the
// whole GPU (deterministic, not bit-identical), so the
// chosen index can differ from the reference's only when r lies within the
// rounding difference of two cumulative sums (about vocab * 2^-24).
#include "common.cuh"
#include "exact_expf.h"

namespace ofb {

constexpr int MV_T = 4;         // tokens per pass
constexpr int MV_THREADS = 256;

template <int TYPE>
__device__ __forceinline__ float mv_weight(const uint8_t *W, uint64_t lin) {
    if (TYPE == OFB_TYPE_F32) return __ldg(reinterpret_cast<const float *>(W) + lin);
    if (TYPE == OFB_TYPE_F16)
        return half_bits_ref(__ldg(reinterpret_cast<const uint16_t *>(W) + lin));
    if (TYPE == OFB_TYPE_Q4_K) return q4k_one(W + (lin / QK) * Q4K_BYTES, (int)(lin % QK));
    return q6k_one(W + (lin / QK) * Q6K_BYTES, (int)(lin % QK));
}

// Thread j of the grid owns output column j for tokens [t0, t0 + nt).
template <int TYPE>
__global__ void __launch_bounds__(MV_THREADS) matvec_kernel(const float *__restrict__ x, int t0, int nt, int in_dim,
                                                            int out_dim, const uint8_t *__restrict__ W,
                                                            float *__restrict__ out) {
    extern __shared__ float xs[];  // [nt][in_dim]
    for (int i = threadIdx.x; i < nt * in_dim; i += blockDim.x) xs[i] = x[(size_t)t0 * in_dim + i];
    __syncthreads();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= out_dim) return;
    float acc[MV_T];
#pragma unroll
    for (int t = 0; t < MV_T; t++) acc[t] = 0.0f;
#pragma unroll 8
    for (int i = 0; i < in_dim; i++) {
        const float w = mv_weight<TYPE>(W, (uint64_t)i * out_dim + j);
#pragma unroll
        for (int t = 0; t < MV_T; t++)
            if (t < nt) acc[t] = __fadd_rn(acc[t], __fmul_rn(xs[t * in_dim + i], w));
    }
#pragma unroll
    for (int t = 0; t < MV_T; t++)
        if (t < nt) out[(size_t)(t0 + t) * out_dim + j] = acc[t];
}

// ---- sampling ----------------------------------------------------------------
// Three launches over chunks of SC_CHUNK logits (one chunk per CTA, so the
// whole GPU streams the row): (1) divided logits and chunk maxima, (2) e_i =
// expf(l_i - max) and chunk sums, (3) one CTA: the total, the first chunk
// whose cumulative probability reaches r, then the first index inside it.
constexpr int SC_THREADS = 256;
constexpr int SC_CHUNK = 1024;
constexpr int SC_PER = SC_CHUNK / SC_THREADS;
constexpr int SP_THREADS = 1024;

__device__ __forceinline__ float block_max_256(float m, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wid] = m;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < SC_THREADS / 32; w++) r = fmaxf(r, red[w]);
    return r;
}

__global__ void __launch_bounds__(SC_THREADS) sample_max_kernel(const float *__restrict__ logits, int V, float temp,
                                                                float *__restrict__ scratch,
                                                                float *__restrict__ cmax) {
    __shared__ float red[SC_THREADS / 32];
    const bool div = temp > 0.0f && temp != 1.0f;
    const int base = blockIdx.x * SC_CHUNK;
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < SC_PER; j++) {
        const int i = base + j * SC_THREADS + threadIdx.x;
        if (i < V) {
            const float l = div ? __fdiv_rn(logits[i], temp) : logits[i];
            scratch[i] = l;
            m = fmaxf(m, l);
        }
    }
    m = block_max_256(m, red);
    if (threadIdx.x == 0) cmax[blockIdx.x] = m;
}

__global__ void __launch_bounds__(SC_THREADS) sample_exp_kernel(int V, int NB, float *__restrict__ scratch,
                                                                const float *__restrict__ cmax,
                                                                float *__restrict__ csum) {
    __shared__ float red[SC_THREADS / 32];
    float m = -INFINITY;
    for (int b = threadIdx.x; b < NB; b += SC_THREADS) m = fmaxf(m, cmax[b]);
    m = block_max_256(m, red);
    __syncthreads();  // red is reused below
    const int base = blockIdx.x * SC_CHUNK;
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < SC_PER; j++) {
        const int i = base + j * SC_THREADS + threadIdx.x;
        if (i < V) {
            const float e = ofb_exact_expf(__fsub_rn(scratch[i], m));
            scratch[i] = e;
            s = __fadd_rn(s, e);
        }
    }
    // fixed-order tree: lanes by xor, then warps in order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < SC_THREADS / 32; w++) t = __fadd_rn(t, red[w]);
        csum[blockIdx.x] = t;
    }
}

// Inclusive scan of v over the 1024 threads (warp shuffles, then warp totals);
// returns this thread's inclusive value and the block total in *total.
__device__ __forceinline__ float block_scan_1024(float v, float *wsum, float *total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v = __fadd_rn(v, u);
    }
    if (lane == 31) wsum[wid] = v;
    __syncthreads();
    if (wid == 0) {
        float w = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w = __fadd_rn(w, u);
        }
        wsum[lane] = w;
    }
    __syncthreads();
    const float r = wid ? __fadd_rn(v, wsum[wid - 1]) : v;
    *total = wsum[31];
    __syncthreads();  // wsum is reused by the next call
    return r;
}

__global__ void __launch_bounds__(SP_THREADS) sample_pick_kernel(int V, int NB, float r,
                                                                 const float *__restrict__ scratch,
                                                                 const float *__restrict__ csum,
                                                                 uint32_t *__restrict__ token) {
    __shared__ float red[SP_THREADS / 32];
    __shared__ float s_sum;
    __shared__ int s_hit;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    float s = 0.0f;
    for (int b = tid; b < NB; b += SP_THREADS) s = __fadd_rn(s, csum[b]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) red[wid] = s;
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int w = 0; w < SP_THREADS / 32; w++) t = __fadd_rn(t, red[w]);
        s_sum = t;
        s_hit = 0x7fffffff;
    }
    __syncthreads();
    const float sum = s_sum;
    // the first chunk whose cumulative probability reaches r
    float carry = 0.0f, prefix = 0.0f;
    int chunk = -1;
    for (int b0 = 0; b0 < NB; b0 += SP_THREADS) {
        const int b = b0 + tid;
        const float v = b < NB ? __fdiv_rn(csum[b], sum) : 0.0f;
        float tot;
        const float inc = __fadd_rn(carry, block_scan_1024(v, red, &tot));
        if (b < NB && inc >= r) atomicMin(&s_hit, b);
        __syncthreads();
        if (s_hit != 0x7fffffff) {
            chunk = s_hit;
            if (b == chunk) red[0] = __fsub_rn(inc, v);  // exclusive prefix of the chunk
            __syncthreads();
            prefix = red[0];
            __syncthreads();
            break;
        }
        carry = __fadd_rn(carry, tot);
    }
    if (chunk < 0) {  // r above every cumulative sum: the reference's last index
        if (tid == 0) *token = (uint32_t)(V - 1);
        return;
    }
    if (tid == 0) s_hit = 0x7fffffff;
    __syncthreads();
    const int i = chunk * SC_CHUNK + tid;
    const float v = i < V ? __fdiv_rn(scratch[i], sum) : 0.0f;
    float tot;
    const float inc = __fadd_rn(prefix, block_scan_1024(v, red, &tot));
    if (i < V && inc >= r) atomicMin(&s_hit, i);
    __syncthreads();
    if (tid == 0) {
        // rounding between the chunk-level and element-level sums can leave r
        // just above the chunk's last element: take that element
        const int last = min(V, (chunk + 1) * SC_CHUNK) - 1;
        *token = (uint32_t)(s_hit != 0x7fffffff ? s_hit : last);
    }
}

}  // namespace ofb

using namespace ofb;

extern "C" int ofb_matvec(const float *x, int n_tokens, int in_dim, int out_dim, const void *w, int w_type,
                          float *out, void *stream) {
    if (n_tokens < 0 || in_dim < 1 || out_dim < 1 || (n_tokens && (!x || !w || !out))) {
        set_error("ofb_matvec: bad arguments");
        return OFB_EINVAL;
    }
    if (w_type != OFB_TYPE_F32 && w_type != OFB_TYPE_F16 && w_type != OFB_TYPE_Q4_K && w_type != OFB_TYPE_Q6_K) {
        set_error("ofb_matvec: weight type %d is not F32/F16/Q4_K/Q6_K", w_type);
        return OFB_EUNSUPPORTED;
    }
    if ((w_type == OFB_TYPE_Q4_K || w_type == OFB_TYPE_Q6_K) && ((uint64_t)in_dim * out_dim) % QK) {
        set_error("ofb_matvec: a block-quantised weight needs in_dim * out_dim to be a multiple of 256");
        return OFB_EINVAL;
    }
    const size_t smem = (size_t)MV_T * in_dim * sizeof(float);
    if (smem > 200 * 1024) { set_error("ofb_matvec: in_dim %d too large", in_dim); return OFB_ETOOLARGE; }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint8_t *W = static_cast<const uint8_t *>(w);
    const dim3 grid((out_dim + MV_THREADS - 1) / MV_THREADS);
    static size_t attr[4][64];
    for (int t0 = 0; t0 < n_tokens; t0 += MV_T) {
        const int nt = n_tokens - t0 < MV_T ? n_tokens - t0 : MV_T;
        const size_t sm = (size_t)nt * in_dim * sizeof(float);
        cudaError_t e = cudaSuccess;
        switch (w_type) {
        case OFB_TYPE_F32:
            e = ensure_dyn_smem(matvec_kernel<OFB_TYPE_F32>, smem, attr[0]);
            matvec_kernel<OFB_TYPE_F32><<<grid, MV_THREADS, sm, s>>>(x, t0, nt, in_dim, out_dim, W, out);
            break;
        case OFB_TYPE_F16:
            e = ensure_dyn_smem(matvec_kernel<OFB_TYPE_F16>, smem, attr[1]);
            matvec_kernel<OFB_TYPE_F16><<<grid, MV_THREADS, sm, s>>>(x, t0, nt, in_dim, out_dim, W, out);
            break;
        case OFB_TYPE_Q4_K:
            e = ensure_dyn_smem(matvec_kernel<OFB_TYPE_Q4_K>, smem, attr[2]);
            matvec_kernel<OFB_TYPE_Q4_K><<<grid, MV_THREADS, sm, s>>>(x, t0, nt, in_dim, out_dim, W, out);
            break;
        default:
            e = ensure_dyn_smem(matvec_kernel<OFB_TYPE_Q6_K>, smem, attr[3]);
            matvec_kernel<OFB_TYPE_Q6_K><<<grid, MV_THREADS, sm, s>>>(x, t0, nt, in_dim, out_dim, W, out);
            break;
        }
        if (e != cudaSuccess) return cuda_status(e, "ofb_matvec smem attribute");
        OFB_CHECK_LAUNCH("ofb_matvec");
    }
    return OFB_OK;
}

extern "C" int ofb_sample(const float *logits, int vocab, float temperature, float r, float *scratch,
                          uint32_t *token, void *stream) {
    if (!logits || !scratch || !token || vocab < 1) { set_error("ofb_sample: bad arguments"); return OFB_EINVAL; }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int NB = (vocab + SC_CHUNK - 1) / SC_CHUNK;
    float *cmax = scratch + vocab, *csum = cmax + NB;
    sample_max_kernel<<<NB, SC_THREADS, 0, s>>>(logits, vocab, temperature, scratch, cmax);
    OFB_CHECK_LAUNCH("ofb_sample max");
    sample_exp_kernel<<<NB, SC_THREADS, 0, s>>>(vocab, NB, scratch, cmax, csum);
    OFB_CHECK_LAUNCH("ofb_sample exp");
    sample_pick_kernel<<<1, SP_THREADS, 0, s>>>(vocab, NB, r, scratch, csum, token);
    OFB_CHECK_LAUNCH("ofb_sample pick");
    return OFB_OK;
}
