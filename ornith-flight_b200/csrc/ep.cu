// ep.cu — expert-parallel dispatch plan, send-buffer packing, combine, and
// the unit-weight RMSNorm of a layer stack. The all-to-all itself is NCCL
// (called by the host between these kernels); these kernels are the device
// side of the exchange: which rows go where, and how the results come back.
#include "common.cuh"
#include "moe.cuh"

namespace ofb {

constexpr int EP_THREADS = 256;

// One block. Assignment a (expert idx[a]) goes to rank idx[a] / epr. Thread
// j takes the contiguous assignment range [j*chunk, (j+1)*chunk); per-rank
// counts of the ranges are scanned across threads, so the slot order is
// grouped by rank and keeps assignment order inside a rank.
__global__ void __launch_bounds__(EP_THREADS) ep_plan_kernel(const uint32_t *__restrict__ idx, int TK, int epr,
                                                             int n_ranks, int32_t *__restrict__ send_counts,
                                                             int32_t *__restrict__ slot_of,
                                                             int32_t *__restrict__ asg_of) {
    __shared__ int cnt[OFB_EP_MAX_RANKS][EP_THREADS + 1];
    __shared__ int base[OFB_EP_MAX_RANKS + 1];
    const int j = threadIdx.x;
    const int chunk = (TK + EP_THREADS - 1) / EP_THREADS;
    const int a0 = min(TK, j * chunk), a1 = min(TK, a0 + chunk);
    int local[OFB_EP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < OFB_EP_MAX_RANKS; r++) local[r] = 0;
    for (int a = a0; a < a1; a++) {
        const int r = (int)(idx[a] / (uint32_t)epr);
#pragma unroll
        for (int q = 0; q < OFB_EP_MAX_RANKS; q++) local[q] += (q == r);
    }
    for (int r = 0; r < n_ranks; r++) cnt[r][j] = local[r];
    __syncthreads();
    // exclusive scan per rank over threads (one warp per rank, serial over
    // 256 entries split into 32 lanes x 8)
    const int warp = j >> 5, lane = j & 31;
    for (int r = warp; r < n_ranks; r += EP_THREADS / 32) {
        int v[EP_THREADS / 32], sum = 0;
#pragma unroll
        for (int i = 0; i < EP_THREADS / 32; i++) {
            v[i] = cnt[r][lane * (EP_THREADS / 32) + i];
            sum += v[i];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        int run = incl - sum;
#pragma unroll
        for (int i = 0; i < EP_THREADS / 32; i++) {
            cnt[r][lane * (EP_THREADS / 32) + i] = run;
            run += v[i];
        }
        if (lane == 31) cnt[r][EP_THREADS] = incl;  // rank total
    }
    __syncthreads();
    if (j == 0) {
        int acc = 0;
        for (int r = 0; r < n_ranks; r++) {
            base[r] = acc;
            send_counts[r] = cnt[r][EP_THREADS];
            acc += cnt[r][EP_THREADS];
        }
    }
    __syncthreads();
    int pos[OFB_EP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < OFB_EP_MAX_RANKS; r++) pos[r] = r < n_ranks ? base[r] + cnt[r][j] : 0;
    for (int a = a0; a < a1; a++) {
        const int r = (int)(idx[a] / (uint32_t)epr);
        int s = 0;
#pragma unroll
        for (int q = 0; q < OFB_EP_MAX_RANKS; q++)
            if (q == r) s = pos[q]++;
        slot_of[a] = s;
        asg_of[s] = a;
    }
}

// One warp per send slot: the token's x row and the {local expert, weight} pair.
__global__ void ep_pack_kernel(const float *__restrict__ x, const uint32_t *__restrict__ idx,
                               const float *__restrict__ w, int TK, int K, int D, int epr,
                               const int32_t *__restrict__ asg_of, float *__restrict__ send_x,
                               int32_t *__restrict__ send_meta) {
    const int lane = threadIdx.x & 31;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < TK; s += (gridDim.x * blockDim.x) >> 5) {
        const int a = asg_of[s], t = a / K;
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * D);
        float4 *dst = reinterpret_cast<float4 *>(send_x + (size_t)s * D);
        for (int c = lane; c < D / 4; c += 32) dst[c] = __ldg(src + c);
        if (lane == 0) {
            const uint32_t e = idx[a];
            send_meta[2 * s] = (int32_t)(e - (e / (uint32_t)epr) * (uint32_t)epr);
            send_meta[2 * s + 1] = __float_as_int(w[a]);
        }
    }
}

// out[t][d] += r, r = sum_k y_back[slot_of[t*K+k]][d] summed in k order
// first, as the reference accumulates routed_out before adding it to the
// stream (engine/src/model.c:1090, :1142).
__global__ void ep_combine_kernel(const float *__restrict__ y_back, const int32_t *__restrict__ slot_of, int T,
                                  int K, int D, float *__restrict__ out) {
    const size_t n4 = (size_t)T * D / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (D / 4)), c = (int)(i % (D / 4));
        float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < K; k++) {
            const float4 y = __ldg(reinterpret_cast<const float4 *>(y_back + (size_t)slot_of[t * K + k] * D) + c);
            r.x += y.x;
            r.y += y.y;
            r.z += y.z;
            r.w += y.w;
        }
        float4 o = reinterpret_cast<float4 *>(out)[i];
        o.x += r.x;
        o.y += r.y;
        o.z += r.z;
        o.w += r.w;
        reinterpret_cast<float4 *>(out)[i] = o;
    }
}

// One warp per row: out = x / sqrt(mean(x^2) + eps).
__global__ void rmsnorm_kernel(const float *__restrict__ x, int T, int D, float eps, float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += (gridDim.x * blockDim.x) >> 5) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * D);
        float ss = 0.f;
        for (int c = lane; c < D / 4; c += 32) {
            const float4 v = src[c];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)D + eps);
        float4 *dst = reinterpret_cast<float4 *>(out + (size_t)t * D);
        for (int c = lane; c < D / 4; c += 32) {
            const float4 v = src[c];
            dst[c] = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
        }
    }
}

}  // namespace ofb

using namespace ofb;

static bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int ofb_ep_plan(const uint32_t *idx, int n_tokens, int top_k, int experts_per_rank, int n_ranks,
                           int32_t *send_counts, int32_t *slot_of_assignment, int32_t *assignment_of_slot,
                           void *stream) {
    if (n_tokens < 0 || top_k < 1 || experts_per_rank < 1 || n_ranks < 1 || n_ranks > OFB_EP_MAX_RANKS ||
        !send_counts || (n_tokens > 0 && (!idx || !slot_of_assignment || !assignment_of_slot))) {
        set_error("ofb_ep_plan: bad arguments");
        return OFB_EINVAL;
    }
    ep_plan_kernel<<<1, EP_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        idx, n_tokens * top_k, experts_per_rank, n_ranks, send_counts, slot_of_assignment, assignment_of_slot);
    OFB_CHECK_LAUNCH("ep plan");
    return OFB_OK;
}

extern "C" int ofb_ep_pack(const float *x, const uint32_t *idx, const float *w, int n_tokens, int top_k,
                           int d_model, int experts_per_rank, const int32_t *assignment_of_slot, float *send_x,
                           int32_t *send_meta, void *stream) {
    if (n_tokens < 0 || top_k < 1 || d_model < 4 || d_model % 4 || experts_per_rank < 1) {
        set_error("ofb_ep_pack: bad arguments");
        return OFB_EINVAL;
    }
    if (n_tokens == 0) return OFB_OK;
    if (!x || !idx || !w || !assignment_of_slot || !send_x || !send_meta || !al16(x) || !al16(send_x)) {
        set_error("ofb_ep_pack: NULL or unaligned pointer");
        return OFB_EINVAL;
    }
    const int TK = n_tokens * top_k;
    ep_pack_kernel<<<grid_for((uint64_t)TK, 8, 148 * 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, idx, w, TK, top_k, d_model, experts_per_rank, assignment_of_slot, send_x, send_meta);
    OFB_CHECK_LAUNCH("ep pack");
    return OFB_OK;
}

extern "C" int ofb_ep_combine(const float *y_back, const int32_t *slot_of_assignment, int n_tokens, int top_k,
                              int d_model, float *out, void *stream) {
    if (n_tokens < 0 || top_k < 1 || d_model < 4 || d_model % 4) {
        set_error("ofb_ep_combine: bad arguments");
        return OFB_EINVAL;
    }
    if (n_tokens == 0) return OFB_OK;
    if (!y_back || !slot_of_assignment || !out || !al16(y_back) || !al16(out)) {
        set_error("ofb_ep_combine: NULL or unaligned pointer");
        return OFB_EINVAL;
    }
    ep_combine_kernel<<<grid_for((uint64_t)n_tokens * d_model / 4, 256, 148 * 8), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(y_back, slot_of_assignment, n_tokens, top_k, d_model,
                                                             out);
    OFB_CHECK_LAUNCH("ep combine");
    return OFB_OK;
}

extern "C" int ofb_rmsnorm(const float *x, int n_tokens, int d_model, float eps, float *out, void *stream) {
    if (n_tokens < 0 || d_model < 4 || d_model % 4 || (n_tokens > 0 && (!x || !out || !al16(x) || !al16(out)))) {
        set_error("ofb_rmsnorm: bad arguments");
        return OFB_EINVAL;
    }
    if (n_tokens == 0) return OFB_OK;
    rmsnorm_kernel<<<grid_for((uint64_t)n_tokens, 8, 148 * 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, n_tokens, d_model, eps, out);
    OFB_CHECK_LAUNCH("rmsnorm");
    return OFB_OK;
}
