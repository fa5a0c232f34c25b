// async.cuh — bulk copies into shared memory completing on mbarriers, bounded
// waits, and tagged 64-bit words for producer/consumer exchange between the
// CTAs of one grid.
//
// Tagged words: a producer publishes a 32-bit value together with a 32-bit
// tag (the launch's epoch) in one aligned 64-bit store; a consumer polls the
// word with 64-bit loads until the tag matches. Value and tag travel in one
// single-copy-atomic access, so no fence is needed between them and the
// consumer needs one L2 round trip once the value is there. Every wait here is
// bounded in time: on expiry it reports failure and the caller records an
// error and carries on to its exit.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace ofb {
namespace ax {

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One arrival that also announces `bytes` of copies completing on this phase.
__device__ __forceinline__ void mbar_arrive_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.b32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for the phase of the given parity; false after `limit_ns`.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_test(b, parity)) return true;
    const unsigned long long t0 = gtime();
    for (uint32_t i = 0;; i++) {
        if (mbar_test(b, parity)) return true;
        if ((i & 63) == 63 && gtime() - t0 > limit_ns) return false;
    }
}

// Bulk copy global -> this CTA's shared memory (addresses 16-byte aligned,
// size a multiple of 16), completing `bytes` on the mbarrier. Not multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// An L2 policy that evicts the lines it fills first: for bytes read once per
// call (routed expert rows), so they do not push hotter data out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's view of global memory (e.g. data acquired from other
// CTAs) before its later async-proxy (bulk copy) reads of it.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- tagged 64-bit words (value in the low half, tag in the high half) ----
__device__ __forceinline__ void put_tagged(unsigned long long *p, uint32_t value, uint32_t tag) {
    const unsigned long long v = ((unsigned long long)tag << 32) | value;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Two consecutive tagged words (16-byte aligned) in one access; each 64-bit
// element is single-copy atomic on its own.
__device__ __forceinline__ void ld_relaxed64x2(const unsigned long long *p, unsigned long long &a,
                                               unsigned long long &b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Polls the pair p[0], p[1] (16-byte aligned) until both tags equal `tag`;
// false (missing values 0) after `limit_ns`. A warp issuing this on
// consecutive pairs reads whole lines per instruction.
__device__ __forceinline__ bool get_tagged2(const unsigned long long *p, uint32_t tag, uint32_t &v0, uint32_t &v1,
                                            unsigned long long limit_ns) {
    unsigned long long a, b;
    ld_relaxed64x2(p, a, b);
    if ((uint32_t)(a >> 32) != tag || (uint32_t)(b >> 32) != tag) {
        const unsigned long long t0 = gtime();
        for (uint32_t i = 0;; i++) {
            ld_relaxed64x2(p, a, b);
            if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag) break;
            if ((i & 15) == 15) {
                if (gtime() - t0 > limit_ns) {
                    v0 = (uint32_t)(a >> 32) == tag ? (uint32_t)a : 0u;
                    v1 = (uint32_t)(b >> 32) == tag ? (uint32_t)b : 0u;
                    return false;
                }
                __nanosleep(32);
            }
        }
    }
    v0 = (uint32_t)a;
    v1 = (uint32_t)b;
    return true;
}

// Polls *p until its tag equals `tag`; returns the value, or 0 and sets *failed
// after `limit_ns`.
__device__ __forceinline__ uint32_t get_tagged(const unsigned long long *p, uint32_t tag,
                                               unsigned long long limit_ns, bool &failed) {
    unsigned long long v = ld_relaxed64(p);
    if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
    const unsigned long long t0 = gtime();
    for (uint32_t i = 0;; i++) {
        v = ld_relaxed64(p);
        if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
        if ((i & 15) == 15) {
            if (gtime() - t0 > limit_ns) {
                failed = true;
                return 0u;
            }
            __nanosleep(32);
        }
    }
}

// Publishes this thread's earlier stores (gpu scope), then adds n to *p.
__device__ __forceinline__ void count_add(unsigned *p, unsigned n) {
    __threadfence();
    atomicAdd(p, n);
}
// Adds n to *p with release semantics (gpu scope): this thread's earlier
// stores are visible to a thread that acquires the new value.
__device__ __forceinline__ void count_add_release(unsigned *p, unsigned n) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(n) : "memory");
}
// Adds n to *p with no ordering: for counts that only say when to look, over
// data that validates itself (tagged words), so the adder need not wait for its
// earlier stores to become visible first.
__device__ __forceinline__ void count_add_relaxed(unsigned *p, unsigned n) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(n) : "memory");
}
// Adds n to *p with acquire-release semantics (gpu scope); returns the old value.
__device__ __forceinline__ unsigned count_add_acq_rel(unsigned *p, unsigned n) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(n) : "memory");
    return old;
}
// Waits until the counter has reached `target` (wrap-around aware); the
// acquire orders the caller's later loads after the counted stores.
__device__ __forceinline__ bool wait_count(const unsigned *p, unsigned target, unsigned long long limit_ns) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if ((int)(v - target) >= 0) return true;
    const unsigned long long t0 = gtime();
    for (;;) {
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if ((int)(v - target) >= 0) return true;
        if (gtime() - t0 > limit_ns) return false;
    }
}

}  // namespace ax
}  // namespace ofb
