// ep_p2p.cu — expert-parallel MoE layer with the exchange done by the GPUs
// themselves over NVLink: no host synchronisation and no collective library
// on the data path.
//
// Every rank of a group allocates one window of device memory and maps the
// windows of all other ranks (CUDA IPC). Window layout (same offsets on every
// rank), seen as the receiver:
//   flags  [2n] u64   count flag of each source rank (rows it sent here, tag),
//                     return flag of each destination rank (results are back)
//   rows   [n][cap]   token rows from each source (bf16 or f32), cap = the
//                     source's maximum assignments (max_tokens * top_k)
//   meta   [n][cap]   int4 {local expert, float bits of weight, source slot, 0}
//   y_back [cap][D]   f32 results of this rank's own assignments, by slot
// A layer on rank r: route own tokens (certified), plan (slots grouped by
// destination), dispatch (rows and meta stored into each destination's
// region r, then a count flag per destination), the shared expert on own
// tokens while peers' rows arrive, receive (wait for every source's count
// flag; rows beyond a source's count get weight 0, which the expert path's
// skip rule drops), routed experts on the n*cap received rows, return (each
// valid result row stored into its source's y_back at the source's slot,
// then a return flag per source), combine (wait for every return flag; sum
// the routed terms in top-k order and add).
// Why a region per source with fixed capacity: the sender needs no offset
// from other senders, so no count exchange precedes the rows; only real rows
// cross NVLink (padding is never sent or read).
// Reuse is safe without extra handshakes: a rank dispatches layer L+1 only
// after its combine of layer L saw every destination's return flag, which a
// destination raises after its experts of layer L read their rows.
// Flags carry the layer's epoch (advanced by every rank per layer call) in
// their upper half. Every wait is bounded (1 s); on expiry the kernel records
// an error bit and continues with zero counts, so no GPU waits forever.
// No TMA or bulk copy touches peer memory: peer accesses are plain stores.
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "moe.cuh"

namespace ofb {

constexpr unsigned long long EP_WAIT_NS = 1000000000ull;  // 1 s

struct EPArgs {
    uint8_t *peer[OFB_EP_MAX_RANKS];
    int n, me, cap, D, K, epr, T, bf16;
    size_t off_flags, off_rows, off_meta, off_yback, row_bytes;
    uint32_t tag;
};

__device__ __forceinline__ unsigned long long ep_gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
    return t;
}
__device__ __forceinline__ void st_flag(uint8_t *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_flag(const uint8_t *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Waits until the flag carries `tag`; returns its low half (0 on expiry).
__device__ __forceinline__ uint32_t wait_flag(const uint8_t *p, uint32_t tag, unsigned *err) {
    unsigned long long v = ld_flag(p);
    if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
    const unsigned long long t0 = ep_gtime();
    for (;;) {
        __nanosleep(128);
        v = ld_flag(p);
        if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
        if (ep_gtime() - t0 > EP_WAIT_NS) {
            atomicOr(err, 1u);
            return 0u;
        }
    }
}

__device__ __forceinline__ uint32_t bf2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

// The last CTA of a grid to pass this point returns true (all other CTAs'
// earlier stores are then visible system-wide); it resets the ticket.
__device__ __forceinline__ bool last_cta(unsigned *ticket) {
    __shared__ int s_last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
        if (s_last) *ticket = 0;
    }
    __syncthreads();
    if (s_last) __threadfence_system();
    return s_last;
}

// Rows and metadata of every slot into the destination's region for this
// rank, then one count flag per destination.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EPArgs a, const float *__restrict__ x,
                                                          const uint32_t *__restrict__ idx,
                                                          const float *__restrict__ w,
                                                          const int32_t *__restrict__ send_counts,
                                                          const int32_t *__restrict__ asg_of, unsigned *ticket) {
    __shared__ int base[OFB_EP_MAX_RANKS];
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int r = 0; r < a.n; r++) { base[r] = acc; acc += send_counts[r]; }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, TK = a.T * a.K;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < TK; s += (gridDim.x * blockDim.x) >> 5) {
        const int as = asg_of[s], t = as / a.K;
        const uint32_t e = idx[as];
        const int dst = (int)(e / (uint32_t)a.epr), pos = s - base[dst];
        const size_t rix = (size_t)a.me * a.cap + pos;
        uint8_t *row = a.peer[dst] + a.off_rows + rix * a.row_bytes;
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * a.D);
        if (a.bf16) {
            uint2 *d2 = reinterpret_cast<uint2 *>(row);
            for (int c = lane; c < a.D / 4; c += 32) {
                const float4 v = __ldg(src + c);
                d2[c] = make_uint2(bf2(v.x, v.y), bf2(v.z, v.w));
            }
        } else {
            float4 *d4 = reinterpret_cast<float4 *>(row);
            for (int c = lane; c < a.D / 4; c += 32) d4[c] = __ldg(src + c);
        }
        if (lane == 0)
            *reinterpret_cast<int4 *>(a.peer[dst] + a.off_meta + rix * 16) =
                make_int4((int)(e - (uint32_t)dst * a.epr), __float_as_int(w[as]), s, 0);
    }
    if (last_cta(ticket) && threadIdx.x < a.n) {
        const int dst = threadIdx.x;
        st_flag(a.peer[dst] + a.off_flags + (size_t)a.me * 8,
                ((unsigned long long)a.tag << 32) | (uint32_t)send_counts[dst]);
    }
}

// Waits for every source's count; row metadata for the expert path (rows past
// a source's count get weight 0 and are skipped there).
__global__ void __launch_bounds__(256) ep_receive_kernel(EPArgs a, int32_t *__restrict__ meta2,
                                                         int32_t *__restrict__ counts, unsigned *err) {
    __shared__ int cnt[OFB_EP_MAX_RANKS];
    const uint8_t *own = a.peer[a.me];
    if (threadIdx.x < a.n) cnt[threadIdx.x] = (int)wait_flag(own + a.off_flags + threadIdx.x * 8, a.tag, err);
    __threadfence_system();
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x < a.n) counts[threadIdx.x] = cnt[threadIdx.x];
    const int rows = a.n * a.cap;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        const int src = r / a.cap, pos = r - src * a.cap;
        int2 m = make_int2(0, 0);
        if (pos < cnt[src]) {
            const int4 v = __ldcg(reinterpret_cast<const int4 *>(own + a.off_meta + (size_t)r * 16));
            m = make_int2(v.x, v.y);
        }
        reinterpret_cast<int2 *>(meta2)[r] = m;
    }
}

// Every valid result row back to its source's y_back slot, then one return
// flag per source.
__global__ void __launch_bounds__(256) ep_return_kernel(EPArgs a, const float *__restrict__ y_rows,
                                                        const int32_t *__restrict__ counts, unsigned *ticket) {
    const int lane = threadIdx.x & 31;
    const uint8_t *own = a.peer[a.me];
    const int rows = a.n * a.cap;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += (gridDim.x * blockDim.x) >> 5) {
        const int src = r / a.cap, pos = r - src * a.cap;
        if (pos >= counts[src]) continue;
        const int slot = __ldcg(reinterpret_cast<const int4 *>(own + a.off_meta + (size_t)r * 16)).z;
        float4 *dst = reinterpret_cast<float4 *>(a.peer[src] + a.off_yback + (size_t)slot * a.D * 4);
        const float4 *s4 = reinterpret_cast<const float4 *>(y_rows + (size_t)r * a.D);
        for (int c = lane; c < a.D / 4; c += 32) dst[c] = __ldcg(s4 + c);
    }
    if (last_cta(ticket) && threadIdx.x < a.n)
        st_flag(a.peer[threadIdx.x] + a.off_flags + (size_t)(a.n + a.me) * 8, (unsigned long long)a.tag << 32);
}

// Waits for every destination's return flag, then out[t] += the routed terms
// summed in top-k order (model.c:1090 then :1142).
__global__ void __launch_bounds__(256) ep_combine_p2p_kernel(EPArgs a, const int32_t *__restrict__ slot_of,
                                                             float *__restrict__ out, unsigned *err) {
    const uint8_t *own = a.peer[a.me];
    if (threadIdx.x < a.n) wait_flag(own + a.off_flags + (size_t)(a.n + threadIdx.x) * 8, a.tag, err);
    __threadfence_system();
    __syncthreads();
    const float *y_back = reinterpret_cast<const float *>(own + a.off_yback);
    const int D = a.D, K = a.K;
    const size_t n4 = (size_t)a.T * D / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (D / 4)), c = (int)(i % (D / 4));
        float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < K; k++) {
            const float4 y = __ldcg(reinterpret_cast<const float4 *>(y_back + (size_t)slot_of[t * K + k] * D) + c);
            r.x += y.x; r.y += y.y; r.z += y.z; r.w += y.w;
        }
        float4 o = reinterpret_cast<float4 *>(out)[i];
        o.x += r.x; o.y += r.y; o.z += r.z; o.w += r.w;
        reinterpret_cast<float4 *>(out)[i] = o;
    }
}

}  // namespace ofb

using namespace ofb;

struct ofb_ep_group {
    ofb_moe_config cfg, loc_cfg;
    int rank, n, max_tokens, cap, epr;
    EPArgs args;
    uint8_t *win;
    size_t win_bytes;
    bool opened[OFB_EP_MAX_RANKS];
    bool connected;
    ofb_workspace *ws_full, *ws_loc;
    uint8_t *scratch;  // idx, w, send_counts, slot_of, asg_of, counts, meta2, y_rows, tickets, err
    uint32_t *idx;
    float *w;
    int32_t *send_counts, *slot_of, *asg_of, *counts, *meta2;
    float *y_rows;
    unsigned *tickets, *err;
    uint32_t epoch;
};

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

extern "C" int ofb_ep_group_create(const ofb_moe_config *cfg, int rank, int n_ranks, int max_tokens_per_rank,
                                   ofb_ep_group **group, void *ipc_handle_out) {
    int st = check_config(cfg);
    if (st) return st;
    if (!group || !ipc_handle_out || n_ranks < 1 || n_ranks > OFB_EP_MAX_RANKS || rank < 0 || rank >= n_ranks ||
        max_tokens_per_rank < 1 || cfg->n_experts % n_ranks || cfg->layout != OFB_LAYOUT_CONTIGUOUS) {
        set_error("ofb_ep_group_create: bad arguments (rank/n_ranks, experts divisible by ranks, contiguous layout)");
        return OFB_EINVAL;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) <= OFB_EP_HANDLE_BYTES, "IPC handle size");
    ofb_ep_group *g = (ofb_ep_group *)calloc(1, sizeof(ofb_ep_group));
    if (!g) { set_error("ofb_ep_group_create: host OOM"); return OFB_ENOMEM; }
    const int D = cfg->d_model, K = cfg->top_k, n = n_ranks;
    g->cfg = *cfg;
    g->rank = rank;
    g->n = n;
    g->max_tokens = max_tokens_per_rank;
    g->cap = max_tokens_per_rank * K;
    g->epr = cfg->n_experts / n;
    g->loc_cfg = *cfg;
    g->loc_cfg.n_experts = g->epr;
    g->loc_cfg.top_k = 1;
    const int rows = n * g->cap;
    // the receiver's batch takes the tensor-core path above the decode-kernel
    // limit: bf16 rows then (that path computes in bf16 anyway), f32 otherwise
    const bool bf16 = rows > gemv_limit(cfg->hidden) && cfg->hidden <= PREFILL_MAX_H;
    EPArgs &a = g->args;
    a.n = n; a.me = rank; a.cap = g->cap; a.D = D; a.K = K; a.epr = g->epr; a.bf16 = bf16;
    a.row_bytes = (size_t)D * (bf16 ? 2 : 4);
    a.off_flags = 0;
    a.off_rows = al256((size_t)2 * n * 8);
    a.off_meta = a.off_rows + al256((size_t)rows * a.row_bytes);
    a.off_yback = a.off_meta + al256((size_t)rows * 16);
    g->win_bytes = a.off_yback + al256((size_t)g->cap * D * 4);
    cudaError_t e = cudaMalloc((void **)&g->win, g->win_bytes);
    if (e == cudaSuccess) e = cudaMemset(g->win, 0, g->win_bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t *)ipc_handle_out, g->win);
    if (e != cudaSuccess) {
        if (g->win) cudaFree(g->win);
        free(g);
        return cuda_status(e, "ofb_ep_group_create: window");
    }
    // own scratch
    size_t off = 0;
    auto take = [&](size_t b) { size_t o = off; off = al256(off + b); return o; };
    const size_t o_idx = take((size_t)g->cap * 4), o_w = take((size_t)g->cap * 4), o_sc = take(n * 4);
    const size_t o_slot = take((size_t)g->cap * 4), o_asg = take((size_t)g->cap * 4), o_cnt = take(n * 4);
    const size_t o_meta2 = take((size_t)rows * 8), o_y = take((size_t)rows * D * 4), o_tk = take(64);
    e = cudaMalloc((void **)&g->scratch, off);
    if (e == cudaSuccess) e = cudaMemset(g->scratch, 0, off);
    if (e != cudaSuccess) {
        cudaFree(g->win);
        free(g);
        return cuda_status(e, "ofb_ep_group_create: scratch");
    }
    g->idx = (uint32_t *)(g->scratch + o_idx);
    g->w = (float *)(g->scratch + o_w);
    g->send_counts = (int32_t *)(g->scratch + o_sc);
    g->slot_of = (int32_t *)(g->scratch + o_slot);
    g->asg_of = (int32_t *)(g->scratch + o_asg);
    g->counts = (int32_t *)(g->scratch + o_cnt);
    g->meta2 = (int32_t *)(g->scratch + o_meta2);
    g->y_rows = (float *)(g->scratch + o_y);
    g->tickets = (unsigned *)(g->scratch + o_tk);
    g->err = g->tickets + 4;
    if ((st = ofb_workspace_create(cfg, max_tokens_per_rank, &g->ws_full)) ||
        (st = ofb_workspace_create(&g->loc_cfg, rows, &g->ws_loc))) {
        if (g->ws_full) ofb_workspace_destroy(g->ws_full);
        cudaFree(g->scratch);
        cudaFree(g->win);
        free(g);
        return st;
    }
    g->args.peer[rank] = g->win;
    *group = g;
    return OFB_OK;
}

extern "C" int ofb_ep_group_connect(ofb_ep_group *g, const void *all_handles) {
    if (!g || !all_handles) { set_error("ofb_ep_group_connect: NULL argument"); return OFB_EINVAL; }
    const uint8_t *h = static_cast<const uint8_t *>(all_handles);
    for (int r = 0; r < g->n; r++) {
        if (r == g->rank || g->opened[r]) continue;
        cudaIpcMemHandle_t hr;
        memcpy(&hr, h + (size_t)r * OFB_EP_HANDLE_BYTES, sizeof(hr));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_status(e, "ofb_ep_group_connect: cudaIpcOpenMemHandle");
        g->args.peer[r] = static_cast<uint8_t *>(p);
        g->opened[r] = true;
    }
    g->connected = true;
    return OFB_OK;
}

// NCCL entry points used for the handle exchange, resolved at run time so the
// library has no link-time dependency on NCCL.
typedef int (*nccl_count_fn)(void *, int *);
typedef int (*nccl_allgather_fn)(const void *, void *, size_t, int, void *, cudaStream_t);

extern "C" int ofb_ep_group_create_nccl(const ofb_moe_config *cfg, void *comm, int max_tokens_per_rank,
                                        ofb_ep_group **group, void *stream) {
    if (!comm || !group) { set_error("ofb_ep_group_create_nccl: NULL argument"); return OFB_EINVAL; }
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) { set_error("ofb_ep_group_create_nccl: libnccl not found"); return OFB_EUNSUPPORTED; }
    nccl_count_fn count = (nccl_count_fn)dlsym(lib, "ncclCommCount");
    nccl_count_fn user_rank = (nccl_count_fn)dlsym(lib, "ncclCommUserRank");
    nccl_allgather_fn allgather = (nccl_allgather_fn)dlsym(lib, "ncclAllGather");
    if (!count || !user_rank || !allgather) { set_error("ofb_ep_group_create_nccl: NCCL symbols missing"); return OFB_EUNSUPPORTED; }
    int n = 0, r = 0;
    if (count(comm, &n) || user_rank(comm, &r)) { set_error("ofb_ep_group_create_nccl: bad communicator"); return OFB_EINVAL; }
    unsigned char h[OFB_EP_HANDLE_BYTES] = {};
    int st = ofb_ep_group_create(cfg, r, n, max_tokens_per_rank, group, h);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *dbuf = nullptr;
    std::vector<uint8_t> all((size_t)n * OFB_EP_HANDLE_BYTES);
    cudaError_t e = cudaMalloc((void **)&dbuf, (size_t)(n + 1) * OFB_EP_HANDLE_BYTES);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dbuf + (size_t)n * OFB_EP_HANDLE_BYTES, h, OFB_EP_HANDLE_BYTES,
                                              cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess &&
        allgather(dbuf + (size_t)n * OFB_EP_HANDLE_BYTES, dbuf, OFB_EP_HANDLE_BYTES, 1 /* ncclUint8 */, comm, s))
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaMemcpyAsync(all.data(), dbuf, all.size(), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (dbuf) cudaFree(dbuf);
    if (e != cudaSuccess) {
        ofb_ep_group_destroy(*group);
        *group = nullptr;
        return cuda_status(e, "ofb_ep_group_create_nccl: handle exchange");
    }
    if ((st = ofb_ep_group_connect(*group, all.data()))) {
        ofb_ep_group_destroy(*group);
        *group = nullptr;
    }
    return st;
}

extern "C" int ofb_ep_group_destroy(ofb_ep_group *g) {
    if (!g) return OFB_OK;
    for (int r = 0; r < g->n; r++)
        if (g->opened[r]) cudaIpcCloseMemHandle(g->args.peer[r]);
    if (g->ws_full) ofb_workspace_destroy(g->ws_full);
    if (g->ws_loc) ofb_workspace_destroy(g->ws_loc);
    cudaFree(g->scratch);
    cudaError_t e = cudaFree(g->win);
    free(g);
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "ofb_ep_group_destroy");
}

extern "C" int ofb_ep_layer_forward(ofb_ep_group *g, const ofb_moe_weights *w, const float *x, const float *resid,
                                    float *out, int n_tokens, void *stream) {
    if (!g || !w || n_tokens < 0 || n_tokens > g->max_tokens) {
        set_error("ofb_ep_layer_forward: bad arguments (n_tokens %d, max %d)", n_tokens, g ? g->max_tokens : 0);
        return OFB_EINVAL;
    }
    if (!g->connected && g->n > 1) { set_error("ofb_ep_layer_forward: group not connected"); return OFB_EINVAL; }
    if (!w->router || !w->gate_exps || !w->up_exps || !w->down_exps || (n_tokens && (!x || !out))) {
        set_error("ofb_ep_layer_forward: NULL tensor");
        return OFB_EINVAL;
    }
    if (x == out) { set_error("ofb_ep_layer_forward: out must not alias x"); return OFB_EINVAL; }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int T = n_tokens, K = g->cfg.top_k, D = g->cfg.d_model;
    EPArgs a = g->args;
    a.T = T;
    a.tag = ++g->epoch;
    int st;
    if (T) {
        if ((st = ofb_route_certified(&g->cfg, w->router, x, T, g->idx, g->w, g->ws_full, stream))) return st;
    }
    if ((st = ofb_ep_plan(g->idx, T, K, g->epr, g->n, g->send_counts, g->slot_of, g->asg_of, stream))) return st;
    ep_dispatch_kernel<<<grid_for((uint64_t)T * K, 8, 148), 256, 0, s>>>(a, x, g->idx, g->w, g->send_counts,
                                                                           g->asg_of, g->tickets);
    OFB_CHECK_LAUNCH("ep dispatch");
    // the shared expert (and the residual) while peers' rows arrive
    if (T) {
        if (w->gate_shexp && w->up_shexp && w->down_shexp) {
            if ((st = ofb_moe_shared(&g->cfg, w, x, resid, out, T, g->ws_full, stream))) return st;
        } else {
            cudaError_t e = resid ? (resid == out ? cudaSuccess
                                                  : cudaMemcpyAsync(out, resid, (size_t)T * D * 4,
                                                                    cudaMemcpyDeviceToDevice, s))
                                  : cudaMemsetAsync(out, 0, (size_t)T * D * 4, s);
            if (e != cudaSuccess) return cuda_status(e, "ofb_ep_layer_forward: out init");
        }
    }
    const int rows = g->n * g->cap;
    ep_receive_kernel<<<grid_for((uint64_t)rows, 256, 148), 256, 0, s>>>(a, g->meta2, g->counts, g->err);
    OFB_CHECK_LAUNCH("ep receive");
    const uint8_t *rbase = g->win + a.off_rows;
    if ((st = run_experts_given(&g->loc_cfg, w, a.bf16 ? nullptr : reinterpret_cast<const float *>(rbase),
                                a.bf16 ? reinterpret_cast<const __nv_bfloat16 *>(rbase) : nullptr, rows, g->meta2,
                                g->y_rows, g->ws_loc, s)))
        return st;
    ep_return_kernel<<<grid_for((uint64_t)rows, 8, 148), 256, 0, s>>>(a, g->y_rows, g->counts, g->tickets + 1);
    OFB_CHECK_LAUNCH("ep return");
    if (T) {
        ep_combine_p2p_kernel<<<grid_for((uint64_t)T * D / 4, 256, 148), 256, 0, s>>>(a, g->slot_of, out, g->err);
    } else {
        // no tokens: still wait for the return flags so the epochs stay in step
        ep_combine_p2p_kernel<<<1, 256, 0, s>>>(a, g->slot_of, out, g->err);
    }
    OFB_CHECK_LAUNCH("ep combine");
    return OFB_OK;
}

extern "C" int ofb_ep_group_device_errors(ofb_ep_group *g, unsigned *bits) {
    if (!g || !bits) { set_error("ofb_ep_group_device_errors: NULL argument"); return OFB_EINVAL; }
    cudaError_t e = cudaMemcpy(bits, g->err, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(g->err, 0, sizeof(unsigned));
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "ofb_ep_group_device_errors");
}
