// exchange.cuh — warp emulation of the reference's exchange sort.
#pragma once
#include "common.cuh"

namespace ofb {

// ---- exchange-sort emulation ---------------------------------------------
// One pass i of "for j>i: if a[j] > a[i] swap" over a[0..n): the holder at i
// is replaced whenever a strictly larger element is met, and the displaced
// holder lands where that element was. Equivalently, with records
// j1<...<jr (positions whose value beats every earlier value in [i, j)):
// a[j1] <- a[i], a[j2] <- a[j1], ..., a[i] <- a[jr]. Records come from a warp
// scan of (value, first position of the running max). `old` holds a copy of
// the arrays taken before the pass.
struct MaxPos { float v; int p; };
__device__ __forceinline__ MaxPos later_if_greater(MaxPos a, MaxPos b) { return (b.v > a.v) ? b : a; }

static __device__ void exchange_pass(float *val, int *id, float *oval, int *oid, int n, int i, int lane) {
    const int per = (n + 31) / 32;
    const int lo = lane * per, hi = min(n, lo + per);
    for (int j = lo; j < hi; j++) { oval[j] = val[j]; oid[j] = id[j]; }
    __syncwarp();
    MaxPos seg = {-INFINITY, -1};
    for (int j = max(lo, i + 1); j < hi; j++) seg = later_if_greater(seg, MaxPos{oval[j], j});
    // inclusive scan over lanes (earlier lanes on the left)
    MaxPos inc = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        MaxPos up;
        up.v = __shfl_up_sync(0xffffffffu, inc.v, o);
        up.p = __shfl_up_sync(0xffffffffu, inc.p, o);
        if (lane >= o) inc = later_if_greater(up, inc);
    }
    MaxPos exc;
    exc.v = __shfl_up_sync(0xffffffffu, inc.v, 1);
    exc.p = __shfl_up_sync(0xffffffffu, inc.p, 1);
    const MaxPos holder = {oval[i], i};
    MaxPos run = (lane == 0) ? holder : later_if_greater(holder, exc);
    for (int j = max(lo, i + 1); j < hi; j++) {
        if (oval[j] > run.v) {
            val[j] = oval[run.p];
            id[j] = oid[run.p];
            run = MaxPos{oval[j], j};
        }
    }
    MaxPos last;
    last.v = __shfl_sync(0xffffffffu, inc.v, 31);
    last.p = __shfl_sync(0xffffffffu, inc.p, 31);
    last = later_if_greater(holder, last);
    if (lane == 0 && last.p != i) { val[i] = oval[last.p]; id[i] = oid[last.p]; }
    __syncwarp();
}

// The first k passes of the reference's exchange sort (engine/src/model.c:
// 1042-1049) over a[0..n), literally, by one thread: for short candidate
// lists this is much faster than k warp passes. Same result as exchange_pass
// for i = 0..k-1.
static __device__ __forceinline__ void exchange_sort_serial(float *val, int *id, int n, int k) {
    for (int i = 0; i < k && i < n; i++) {
        float vi = val[i];
        int ii = id[i];
        for (int j = i + 1; j < n; j++) {
            const float vj = val[j];
            if (vj > vi) {
                val[j] = vi;
                const int ij = id[j];
                id[j] = ii;
                vi = vj;
                ii = ij;
            }
        }
        val[i] = vi;
        id[i] = ii;
    }
}

// Top-k passes over n candidates by warp `lane`s: serial for short lists,
// else the warp emulation.
constexpr int EXCHANGE_SERIAL_MAX = 64;
static __device__ __forceinline__ void exchange_topk(float *val, int *id, float *oval, int *oid, int n, int k,
                                                     int lane) {
    if (n <= EXCHANGE_SERIAL_MAX) {
        if (lane == 0) exchange_sort_serial(val, id, n, k);
        __syncwarp();
    } else {
        for (int i = 0; i < k; i++) exchange_pass(val, id, oval, oid, n, i, lane);
    }
}

}  // namespace ofb
