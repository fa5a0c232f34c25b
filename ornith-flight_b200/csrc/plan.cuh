// plan.cuh — device construction of the per-expert dispatch plan.
#pragma once
#include "common.cuh"
#include "moe.cuh"

namespace ofb {

// ---- plan ------------------------------------------------------------------
// Device histogram of kept assignments per expert, exclusive scan, and the
// CSR slot list. Works for any block size (E <= 1024); scratch in `sm`
// (2*1024 ints + 64). Called by the last block of
// the fast routing kernel (small T).
static __device__ void build_plan(const PlanArgs &p, int *cnt, int *cursor, int *wsum) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5, nw = nt >> 5;
    const int TK = p.T * p.K;
    for (int e = tid; e < p.E; e += nt) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < TK; i += nt) {
        float wv = __ldcg(p.w + i);
        if (!(wv < 1e-6f)) atomicAdd(&cnt[__ldcg(p.idx + i)], 1);  // model.c:1066 skip rule
    }
    __syncthreads();
    // each thread owns a run of `per` consecutive experts
    const int per = (p.E + nt - 1) / nt, e0 = tid * per, e1 = min(p.E, e0 + per);
    int f = 0, c = 0;
    for (int e = e0; e < e1; e++) { f += cnt[e] > 0; c += cnt[e]; }
    int fi = f, ci = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int nf = __shfl_up_sync(0xffffffffu, fi, o), nc = __shfl_up_sync(0xffffffffu, ci, o);
        if (lane >= o) { fi += nf; ci += nc; }
    }
    if (lane == 31) { wsum[2 * wid] = fi; wsum[2 * wid + 1] = ci; }
    __syncthreads();
    if (wid == 0) {
        int a = lane < nw ? wsum[2 * lane] : 0, b = lane < nw ? wsum[2 * lane + 1] : 0;
        int ai = a, bi = b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int na = __shfl_up_sync(0xffffffffu, ai, o), nb = __shfl_up_sync(0xffffffffu, bi, o);
            if (lane >= o) { ai += na; bi += nb; }
        }
        if (lane < nw) { wsum[2 * lane] = ai - a; wsum[2 * lane + 1] = bi - b; }
        if (lane == nw - 1) { wsum[64] = ai; wsum[65] = bi; }
    }
    __syncthreads();
    int F = fi - f + wsum[2 * wid], C = ci - c + wsum[2 * wid + 1];
    for (int e = e0; e < e1; e++) {
        if (cnt[e] > 0) { p.slot_expert[F] = e; p.slot_start[F] = C; F++; }
        cursor[e] = C;
        C += cnt[e];
    }
    if (tid == 0) {
        const int nslots = wsum[64], total = wsum[65];
        int u = nslots;
        if (p.has_shared) {
            p.slot_expert[u] = p.E;
            p.slot_start[u] = total;
            u++;
            p.slot_start[u] = total + p.T;
        } else {
            p.slot_start[u] = total;
        }
        *p.n_slots = u;
    }
    if (p.has_shared)
        for (int t = tid; t < p.T; t += nt) p.assign[wsum[65] + t] = TK + t;
    __syncthreads();
    for (int i = tid; i < TK; i += nt) {
        float wv = __ldcg(p.w + i);
        if (!(wv < 1e-6f)) p.assign[atomicAdd(&cursor[__ldcg(p.idx + i)], 1)] = i;
    }
}

}  // namespace ofb
