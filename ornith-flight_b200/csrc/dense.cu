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
// sums are a fixed-order tree (deterministic, not bit-identical), so the
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
constexpr int SM_THREADS = 1024;

__global__ void __launch_bounds__(SM_THREADS) sample_kernel(const float *__restrict__ logits, int V, float temp,
                                                            float r, float *__restrict__ scratch,
                                                            uint32_t *__restrict__ token) {
    __shared__ float red[SM_THREADS / 32];
    __shared__ float s_max, s_sum;
    __shared__ float part[SM_THREADS];
    __shared__ int s_tok;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const bool div = temp > 0.0f && temp != 1.0f;
    // max of the (divided) logits
    float m = -INFINITY;
    for (int i = tid; i < V; i += SM_THREADS) {
        const float l = div ? __fdiv_rn(logits[i], temp) : logits[i];
        scratch[i] = l;
        m = fmaxf(m, l);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wid] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < SM_THREADS / 32; w++) mm = fmaxf(mm, red[w]);
        s_max = mm;
    }
    __syncthreads();
    // e_i = expf(l_i - max) (the host library's function); thread tid owns the
    // contiguous chunk [tid*per, tid*per + per), summed in order
    const int per = (V + SM_THREADS - 1) / SM_THREADS;
    const int a = min(V, tid * per), b = min(V, a + per);
    float s = 0.0f;
    for (int i = a; i < b; i++) {
        const float e = ofb_exact_expf(__fsub_rn(scratch[i], s_max));
        scratch[i] = e;
        s = __fadd_rn(s, e);
    }
    part[tid] = s;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.0f;
        for (int w = 0; w < SM_THREADS; w++) tot = __fadd_rn(tot, part[w]);
        s_sum = tot;
        s_tok = V - 1;
    }
    __syncthreads();
    // cumulative probability: chunk prefix (one thread), then inside the
    // chunk; the first index whose cumulative sum reaches r
    if (tid == 0) {
        float c = 0.0f;
        for (int w = 0; w < SM_THREADS; w++) {
            const float nc = __fadd_rn(c, __fdiv_rn(part[w], s_sum));
            part[w] = c;  // exclusive prefix of chunk w
            c = nc;
        }
    }
    __syncthreads();
    float cum = part[tid];
    int found = 0x7fffffff;
    for (int i = a; i < b; i++) {
        cum = __fadd_rn(cum, __fdiv_rn(scratch[i], s_sum));
        if (cum >= r) { found = i; break; }
    }
    atomicMin(&s_tok, found);
    __syncthreads();
    if (tid == 0) *token = (uint32_t)s_tok;
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
    sample_kernel<<<1, SM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(logits, vocab, temperature, r, scratch,
                                                                           token);
    OFB_CHECK_LAUNCH("ofb_sample");
    return OFB_OK;
}
