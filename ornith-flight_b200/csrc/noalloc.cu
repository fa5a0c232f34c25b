// noalloc.cu — ofb_moe_forward_noalloc: the MoE layer forward without any
// device allocation, for callers that cannot call cudaMalloc.
//
// Who cannot allocate: an engine whose device memory is reserved up front by
// its own pool or budget (the reference engine sizes all of its memory from a
// fixed budget at start-up, engine/src/memory.c:397-421; embedders such as a
// PyTorch process keep HBM in a caching allocator), where a raw cudaMalloc
// can fail or take memory the owner has already promised elsewhere; and
// per-token decode loops, where cudaMalloc/cudaFree would synchronise the
// device inside the latency-critical step.
//
// The scratch the layer needs (routing logits and bounds, dispatch plan,
// quantised activations, expert intermediates, combine tickets) lives in the
// file-scope device array below, of a fixed size: every GPU that loads this
// library holds it until the process exits. Host code must not pass the
// array's name to a kernel (on the host it names a host-side stand-in, not a
// device address); the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, by the first call made on
// that device. Make that first call before any stream capture. The address
// is remembered together with the device's current context; if the context
// changes (cudaDeviceReset, then a new primary context), the next call looks
// the address up again.
//
// All calls share the one array and every call overwrites it, so calls
// whose GPU work overlaps in time (on different streams, or from different
// host threads) race and give wrong results; calls in one stream are safe.
// Each call clears the ticket counters that must start at zero.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "moe.cuh"

// Maximum scratch of one call (the layer's workspace size must not exceed it).
#define OFB_NOALLOC_SCRATCH_BYTES (8u << 20)

static __device__ __align__(256) unsigned char ofb_noalloc_scratch[OFB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
uint8_t *g_scratch_ptr[kMaxDevices];
CUcontext g_scratch_ctx[kMaxDevices];
std::mutex g_scratch_mu;

int scratch_for_current_device(uint8_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return ofb::cuda_status(e, "noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        ofb::set_error("noalloc: device ordinal %d beyond %d", dev, kMaxDevices);
        return OFB_EUNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    // the device's current context, through the runtime's driver entry
    // point (the library does not link the driver library directly)
    using CtxGetCurrentFn = CUresult (*)(CUcontext *);
    static CtxGetCurrentFn ctx_get = nullptr;
    if (!ctx_get) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ctx_get = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    CUcontext ctx = nullptr;
    if (!ctx_get || ctx_get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, ofb_noalloc_scratch);
        if (e != cudaSuccess || !p) return ofb::cuda_status(e, "noalloc: cudaGetSymbolAddress");
        // the single-launch decode keeps an epoch and tagged words at the
        // start of the scratch across calls: they start from zero once
        e = cudaMemset(p, 0, OFB_NOALLOC_SCRATCH_BYTES);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return ofb::cuda_status(e, "noalloc: scratch set-up");
        g_scratch_ptr[dev] = static_cast<uint8_t *>(p);
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_ptr[dev];
    return OFB_OK;
}
}  // namespace

extern "C" size_t ofb_noalloc_capacity(void) { return OFB_NOALLOC_SCRATCH_BYTES; }

extern "C" int ofb_moe_forward_noalloc(const ofb_moe_config *cfg, const ofb_moe_weights *w,
                                       const float *x, const float *resid, float *out, int n_tokens,
                                       uint32_t *idx_out, float *w_out, void *stream) {
    using namespace ofb;
    int st = check_config(cfg);
    if (st) return st;
    if (!w || n_tokens < 0) { set_error("ofb_moe_forward_noalloc: bad arguments"); return OFB_EINVAL; }
    if (n_tokens == 0) return OFB_OK;
    if (!x || !out || !w->gate_exps || !w->up_exps || !w->down_exps) {
        set_error("ofb_moe_forward_noalloc: NULL tensor");
        return OFB_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(w->gate_exps) | reinterpret_cast<uintptr_t>(w->up_exps) |
         reinterpret_cast<uintptr_t>(w->down_exps) | reinterpret_cast<uintptr_t>(w->gate_shexp) |
         reinterpret_cast<uintptr_t>(w->up_shexp) | reinterpret_cast<uintptr_t>(w->down_shexp) |
         reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w->router)) & 15) {
        set_error("ofb_moe_forward_noalloc: tensors must be 16-byte aligned");
        return OFB_EINVAL;
    }
    const WorkspaceLayout L = workspace_layout(cfg, n_tokens);
    if (L.total > OFB_NOALLOC_SCRATCH_BYTES) {
        set_error("ofb_moe_forward_noalloc: %d tokens of this layer need %zu bytes of scratch, more than "
                  "the fixed %u; use ofb_moe_forward with a workspace, or fewer tokens per call",
                  n_tokens, L.total, (unsigned)OFB_NOALLOC_SCRATCH_BYTES);
        return OFB_ETOOLARGE;
    }
    uint8_t *base = nullptr;
    if ((st = scratch_for_current_device(&base))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // tickets and counters must start at zero; a finished call leaves them
    // zero, an interrupted one might not
    cudaError_t e = cudaMemsetAsync(base + L.counters, 0, L.counters_bytes, s);
    if (e != cudaSuccess) return cuda_status(e, "noalloc: clear counters");
    return run_moe_layer(cfg, w, x, resid, out, n_tokens, idx_out, w_out, base, L, s, nullptr);
}
