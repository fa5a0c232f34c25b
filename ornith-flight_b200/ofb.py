"""Python binding of libornith_cuda.so (the C ABI in include/ornith_moe.h).

Host-side mirror of the reference's MoE-path interfaces for the test and
benchmark harness. Device memory and streams come from PyTorch (plumbing
only); every computation runs in the CUDA library. There is no CPU path:
if the library is missing, loading this module raises.

Reference interfaces mirrored (ornith-flight, file:line):
  dequantize           gguf_dequantize_tensor_from_buf   engine/src/gguf.c:605-638
  dequantize_slice     gguf_dequantize_expert_slice_from_buf  engine/src/gguf.c:652-711
  route                model_get_routing / inline router  engine/src/model.c:264-321, :1017-1049
  MoeLayer.forward     MoE block of model_forward         engine/src/model.c:992-1143
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libornith_cuda.so")

OK, EINVAL, ECUDA, ENOMEM, EUNSUPPORTED, ETOOLARGE = range(6)
TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 12, 14
OUT_F32, OUT_BF16 = 0, 1
LAYOUT_CONTIGUOUS, LAYOUT_INTERLEAVED = 0, 1
ROUTE_FORWARD, ROUTE_GET_ROUTING = 0, 1
QK = 256
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210}


class OfbError(RuntimeError):
    def __init__(self, status: int, detail: str):
        super().__init__(f"ornith-flight-b200 status {status}: {detail}")
        self.status = status


class MoeConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "d_model", "hidden", "n_experts", "top_k", "layout", "routing", "renorm", "shared_gate")]


class MoeWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
        "shexp_gate")]


class GgufMoeLayer(ctypes.Structure):
    """ofb_gguf_moe_layer: config read from the file + device weight pointers."""
    _fields_ = [("cfg", MoeConfig), ("weights", MoeWeights)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `make -C {_HERE}` (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    vp, u64, i32, sz = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t
    cfgp, wp = ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights)
    sig = {
        "ofb_status_string": (ctypes.c_char_p, [i32]),
        "ofb_last_error": (ctypes.c_char_p, []),
        "ofb_build_info": (ctypes.c_char_p, []),
        "ofb_dequantize": (i32, [vp, i32, u64, vp, i32, vp]),
        "ofb_dequantize_expert_slice": (i32, [vp, i32, u64, u64, i32, vp, i32, vp]),
        "ofb_route": (i32, [cfgp, vp, vp, i32, vp, vp, vp, vp]),
        "ofb_route_certified": (i32, [cfgp, vp, vp, i32, vp, vp, vp, vp]),
        "ofb_workspace_size": (sz, [cfgp, i32]),
        "ofb_workspace_create": (i32, [cfgp, i32, ctypes.POINTER(vp)]),
        "ofb_workspace_destroy": (i32, [vp]),
        "ofb_moe_forward": (i32, [cfgp, wp, vp, vp, vp, i32, vp, vp, vp, vp]),
        "ofb_moe_forward_profiled": (i32, [cfgp, wp, vp, vp, vp, i32, vp, vp, vp]),
        "ofb_workspace_route_stats": (i32, [vp, ctypes.POINTER(ctypes.c_int * 3)]),
        "ofb_workspace_device_errors": (i32, [vp, ctypes.POINTER(ctypes.c_uint)]),
        "ofb_moe_forward_noalloc": (i32, [cfgp, wp, vp, vp, vp, i32, vp, vp, vp]),
        "ofb_noalloc_capacity": (sz, []),
        "ofb_synth_blocks": (i32, [vp, i32, u64, u64, u64, u64, vp]),
        "ofb_synth_blocks_host": (None, [vp, i32, u64, u64, u64, u64]),
        "ofb_synth_normal_host": (None, [vp, u64, u64, u64, ctypes.c_float]),
        "ofb_ep_plan": (i32, [vp, i32, i32, i32, i32, vp, vp, vp, vp]),
        "ofb_ep_pack": (i32, [vp, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp]),
        "ofb_moe_experts": (i32, [cfgp, wp, vp, i32, vp, vp, vp, vp]),
        "ofb_moe_shared": (i32, [cfgp, wp, vp, vp, vp, i32, vp, vp]),
        "ofb_ep_combine": (i32, [vp, vp, i32, i32, i32, vp, vp]),
        "ofb_rmsnorm": (i32, [vp, i32, i32, ctypes.c_float, vp, vp]),
        "ofb_copy": (i32, [vp, vp, sz, vp]),
        "ofb_matvec": (i32, [vp, i32, i32, i32, vp, i32, vp, vp]),
        "ofb_sample": (i32, [vp, i32, ctypes.c_float, ctypes.c_float, vp, vp, vp]),
        "ofb_gguf_open": (i32, [ctypes.c_char_p, ctypes.POINTER(vp)]),
        "ofb_gguf_close": (i32, [vp]),
        "ofb_gguf_tensor": (i32, [vp, ctypes.c_char_p, ctypes.POINTER(i32), ctypes.POINTER(i32),
                                  ctypes.POINTER(ctypes.c_uint64 * 4), ctypes.POINTER(u64), ctypes.POINTER(u64)]),
        "ofb_gguf_param_u32": (i32, [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]),
        "ofb_gguf_upload": (i32, [vp, ctypes.c_char_p, vp, u64, vp]),
        "ofb_gguf_upload_moe_layer": (i32, [vp, i32, i32, vp, vp]),
        "ofb_gguf_free_moe_layer": (i32, [vp]),
        "ofb_ep_group_create": (i32, [cfgp, i32, i32, i32, ctypes.POINTER(vp), vp]),
        "ofb_ep_group_connect": (i32, [vp, vp]),
        "ofb_ep_group_create_nccl": (i32, [cfgp, vp, i32, ctypes.POINTER(vp), vp]),
        "ofb_ep_group_destroy": (i32, [vp]),
        "ofb_ep_layer_forward": (i32, [vp, wp, vp, vp, vp, i32, vp]),
        "ofb_ep_group_device_errors": (i32, [vp, ctypes.POINTER(ctypes.c_uint)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# Entry points declared in include/*.h that the library must export.
EXPORTED = [
    "ofb_status_string", "ofb_last_error", "ofb_build_info", "ofb_dequantize",
    "ofb_dequantize_expert_slice", "ofb_route", "ofb_workspace_size", "ofb_workspace_create",
    "ofb_workspace_destroy", "ofb_moe_forward", "ofb_moe_forward_profiled", "ofb_workspace_route_stats",
    "ofb_workspace_device_errors", "ofb_synth_blocks", "ofb_synth_blocks_host",
    "ofb_synth_normal_host",
]


def _check(status: int) -> None:
    if status != OK:
        raise OfbError(status, lib.ofb_last_error().decode())


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def decode_path(n_rows: int, hidden: int) -> bool:
    """True when a batch of n_rows token rows runs on the fp32-accumulating
    dp4a decode kernels (tolerance 1e-3), False on the bf16 tensor-core
    kernels (2e-2); the library's dispatch rule (moe.cuh use_gemv)."""
    return n_rows <= (4 if hidden <= 512 else 32)


# ---- dequant ----------------------------------------------------------------

def dequantize(blocks: torch.Tensor, qtype: int, n_elems: int, out_dtype=torch.float32,
               out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Whole-tensor decode of device `blocks` (uint8) to f32 or bf16."""
    if out is None:
        out = torch.empty(n_elems, dtype=out_dtype, device=blocks.device)
    ot = OUT_F32 if out.dtype == torch.float32 else OUT_BF16
    _check(lib.ofb_dequantize(_ptr(blocks), qtype, n_elems, _ptr(out), ot, _stream(stream)))
    return out


def dequantize_slice(blocks: torch.Tensor, qtype: int, n_elems: int, n_experts: int, expert: int,
                     out_dtype=torch.float32, stream=None) -> torch.Tensor:
    """Expert slice with the expert index fastest-varying (reference semantics)."""
    out = torch.empty(n_elems // max(n_experts, 1), dtype=out_dtype, device=blocks.device)
    ot = OUT_F32 if out_dtype == torch.float32 else OUT_BF16
    _check(lib.ofb_dequantize_expert_slice(_ptr(blocks), qtype, n_elems, n_experts, expert,
                                           _ptr(out), ot, _stream(stream)))
    return out


# ---- dense projections and sampling ---------------------------------------------

def copy(dst: torch.Tensor, src: torch.Tensor, stream=None) -> torch.Tensor:
    """dst <- src by a kernel; either may be pinned host memory (ofb_copy)."""
    assert dst.numel() * dst.element_size() == src.numel() * src.element_size()
    _check(lib.ofb_copy(_ptr(dst), _ptr(src), src.numel() * src.element_size(), _stream(stream)))
    return dst


def matvec(x: torch.Tensor, w: torch.Tensor, w_type: int, out_dim: int, stream=None) -> torch.Tensor:
    """out[t][j] = sum_i x[t][i] * W[i*out_dim + j] for a GGUF-typed W (bit-exact)."""
    T, in_dim = x.shape
    out = torch.empty(T, out_dim, dtype=torch.float32, device=x.device)
    _check(lib.ofb_matvec(_ptr(x), T, in_dim, out_dim, _ptr(w), w_type, _ptr(out), _stream(stream)))
    return out


def sample_scratch(vocab: int) -> int:
    """Floats of scratch ofb_sample needs (OFB_SAMPLE_SCRATCH)."""
    return vocab + 2 * ((vocab + 1023) // 1024)


def sample(logits: torch.Tensor, temperature: float, r: float, stream=None) -> int:
    V = logits.numel()
    scratch = torch.empty(sample_scratch(V), dtype=torch.float32, device=logits.device)
    tok = torch.empty(1, dtype=torch.int32, device=logits.device)
    _check(lib.ofb_sample(_ptr(logits), logits.numel(), temperature, r, _ptr(scratch), _ptr(tok), _stream(stream)))
    return int(tok.item())


# ---- synthetic inputs ---------------------------------------------------------

def synth_blocks(qtype: int, n_blocks: int, seed: int, stream_id: int, device="cuda",
                 first_block: int = 0) -> torch.Tensor:
    t = torch.empty(n_blocks * BLOCK_BYTES[qtype], dtype=torch.uint8, device=device)
    _check(lib.ofb_synth_blocks(_ptr(t), qtype, n_blocks, first_block, seed, stream_id, _stream()))
    return t


def synth_blocks_host(qtype: int, n_blocks: int, seed: int, stream_id: int,
                      first_block: int = 0) -> torch.Tensor:
    t = torch.empty(n_blocks * BLOCK_BYTES[qtype], dtype=torch.uint8)
    lib.ofb_synth_blocks_host(_ptr(t), qtype, n_blocks, first_block, seed, stream_id)
    return t


def synth_normal(n: int, seed: int, stream_id: int, sigma: float) -> torch.Tensor:
    t = torch.empty(n, dtype=torch.float32)
    lib.ofb_synth_normal_host(_ptr(t), n, seed, stream_id, sigma)
    return t


# ---- the MoE layer --------------------------------------------------------------

@dataclass
class LayerShape:
    d_model: int = 2048
    hidden: int = 512
    n_experts: int = 256
    top_k: int = 8
    layout: int = LAYOUT_CONTIGUOUS
    routing: int = ROUTE_FORWARD
    renorm: int = 1
    shared_gate: int = 1

    def config(self) -> MoeConfig:
        return MoeConfig(self.d_model, self.hidden, self.n_experts, self.top_k, self.layout,
                         self.routing, self.renorm, self.shared_gate)

    @property
    def q4k_blocks_per_expert(self) -> int:
        return self.hidden * self.d_model // QK

    def expert_bytes(self) -> int:
        nb = self.q4k_blocks_per_expert
        return 2 * nb * 144 + nb * 210


# Generator stream ids of one layer's tensors (seeded per layer).
STREAM_GATE, STREAM_UP, STREAM_DOWN, STREAM_GATE_SH, STREAM_UP_SH, STREAM_DOWN_SH = 1, 2, 3, 4, 5, 6
STREAM_ROUTER, STREAM_GATE_V, STREAM_X = 7, 8, 9


@dataclass
class LayerWeights:
    """One layer's tensors (device or host): raw Q4_K/Q6_K bytes and f32."""
    router: torch.Tensor | None
    gate_exps: torch.Tensor
    up_exps: torch.Tensor
    down_exps: torch.Tensor
    gate_shexp: torch.Tensor | None
    up_shexp: torch.Tensor | None
    down_shexp: torch.Tensor | None
    shexp_gate: torch.Tensor | None

    def struct(self) -> MoeWeights:
        return MoeWeights(*(_ptr(t) for t in (
            self.router, self.gate_exps, self.up_exps, self.down_exps, self.gate_shexp,
            self.up_shexp, self.down_shexp, self.shexp_gate)))

    def to(self, device) -> "LayerWeights":
        return LayerWeights(*(None if t is None else t.to(device) for t in (
            self.router, self.gate_exps, self.up_exps, self.down_exps, self.gate_shexp,
            self.up_shexp, self.down_shexp, self.shexp_gate)))


def make_router(shape: LayerShape, seed: int, router_bias: torch.Tensor | None = None) -> torch.Tensor:
    """Host f32 router of make_layer (flat, laid out per `shape.layout`)."""
    E, D = shape.n_experts, shape.d_model
    r = synth_normal(E * D, seed, STREAM_ROUTER, 0.02).view(E, D)
    if router_bias is not None:
        r[:, 0] = router_bias.float()
    if shape.layout == LAYOUT_INTERLEAVED:
        r = r.t().contiguous()
    return r.reshape(-1)


def make_layer(shape: LayerShape, seed: int, device="cuda", shared: bool = True,
               router: bool = True, router_bias: torch.Tensor | None = None) -> LayerWeights:
    """Seeded synthetic layer with the benchmark's distributions.

    router f32 N(0, 0.02), laid out per `shape.layout`; shared-expert gate
    vector N(0, 0.02); Q4_K/Q6_K blocks from the counter generator (uniform
    quant/scale bytes, d/dmin = fp16(U(0, 0.01))). Blocks are generated on
    `device` (host generator when device is "cpu"; both give the same bytes).
    `router_bias` (f32 [E]) is folded into input coordinate 0 of the router:
    W[e][0] = bias[e] (the inputs set x[:, 0] = 1), which skews routing
    without adding a term the reference does not have.
    """
    E, D, H = shape.n_experts, shape.d_model, shape.hidden
    nb = shape.q4k_blocks_per_expert
    gen = (lambda q, n, s: synth_blocks_host(q, n, seed, s)) if str(device) == "cpu" else \
          (lambda q, n, s: synth_blocks(q, n, seed, s, device=device))
    r = make_router(shape, seed, router_bias).to(device) if router else None
    g = gen(TYPE_Q4_K, E * nb, STREAM_GATE)
    u = gen(TYPE_Q4_K, E * nb, STREAM_UP)
    d = gen(TYPE_Q6_K, E * nb, STREAM_DOWN)
    gs = us = ds = v = None
    if shared:
        gs = gen(TYPE_Q4_K, nb, STREAM_GATE_SH)
        us = gen(TYPE_Q4_K, nb, STREAM_UP_SH)
        ds = gen(TYPE_Q6_K, nb, STREAM_DOWN_SH)
        v = synth_normal(D, seed, STREAM_GATE_V, 0.02).to(device)
    return LayerWeights(r, g, u, d, gs, us, ds, v)


def make_layer_slice(shape: LayerShape, seed: int, e0: int, e1: int, device="cuda",
                     shared: bool = True, router: bool = True) -> LayerWeights:
    """The tensors of make_layer(shape, seed) that one expert-parallel rank
    holds: routed experts [e0, e1) (the same bytes as those experts of the
    whole layer), the full router, the shared expert and its gate vector."""
    nb = shape.q4k_blocks_per_expert
    n = (e1 - e0) * nb
    if str(device) == "cpu":
        gen = lambda q, s: synth_blocks_host(q, n, seed, s, first_block=e0 * nb)
    else:
        gen = lambda q, s: synth_blocks(q, n, seed, s, device=device, first_block=e0 * nb)
    r = make_router(shape, seed).to(device) if router else None
    gs = us = ds = v = None
    if shared:
        sgen = (lambda q, s: synth_blocks_host(q, nb, seed, s)) if str(device) == "cpu" else \
               (lambda q, s: synth_blocks(q, nb, seed, s, device=device))
        gs, us, ds = sgen(TYPE_Q4_K, STREAM_GATE_SH), sgen(TYPE_Q4_K, STREAM_UP_SH), sgen(TYPE_Q6_K, STREAM_DOWN_SH)
        v = synth_normal(shape.d_model, seed, STREAM_GATE_V, 0.02).to(device)
    return LayerWeights(r, gen(TYPE_Q4_K, STREAM_GATE), gen(TYPE_Q4_K, STREAM_UP),
                        gen(TYPE_Q6_K, STREAM_DOWN), gs, us, ds, v)


ZIPF_ALPHA = 0.15  # gives per-expert counts of ~60..600 at 4096 tokens, top-8 of 256


def zipf_bias(n_experts: int, seed: int, alpha: float = ZIPF_ALPHA) -> torch.Tensor:
    """Router logit bias alpha * log(r_e^-1.1) over a seeded expert ranking r
    (the prefill configuration's Zipf(1.1) skew)."""
    g = torch.Generator().manual_seed(seed)
    rank = torch.randperm(n_experts, generator=g).double() + 1.0
    return (alpha * (-1.1) * torch.log(rank)).float()


def make_tokens(shape: LayerShape, n_tokens: int, seed: int, bias_coordinate: bool = False) -> torch.Tensor:
    """Host f32 [T][D] drawn N(0, 1); x[:, 0] = 1 when a router bias is used."""
    x = synth_normal(n_tokens * shape.d_model, seed, STREAM_X, 1.0).view(n_tokens, shape.d_model)
    if bias_coordinate:
        x[:, 0] = 1.0
    return x


class Workspace:
    def __init__(self, shape: LayerShape, max_tokens: int):
        self.shape = shape
        self.max_tokens = max_tokens
        self._cfg = shape.config()
        h = ctypes.c_void_p()
        _check(lib.ofb_workspace_create(ctypes.byref(self._cfg), max_tokens, ctypes.byref(h)))
        self.handle = h

    def route_stats(self):
        """(certified, candidate recompute, full recompute) token counts."""
        c = (ctypes.c_int * 3)()
        _check(lib.ofb_workspace_route_stats(self.handle, ctypes.byref(c)))
        return tuple(c)

    def device_errors(self) -> int:
        """Bits of device-side wait expiries since the last call (0: none)."""
        b = ctypes.c_uint()
        _check(lib.ofb_workspace_device_errors(self.handle, ctypes.byref(b)))
        return b.value

    def close(self):
        if self.handle:
            _check(lib.ofb_workspace_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoeLayer:
    """One MoE feed-forward layer resident in HBM (model.c:992-1143)."""

    def __init__(self, shape: LayerShape, weights: LayerWeights, max_tokens: int):
        self.shape = shape
        self.weights = weights
        self._cfg = shape.config()
        self._w = weights.struct()
        self.ws = Workspace(shape, max_tokens)

    def forward(self, x: torch.Tensor, resid: torch.Tensor | None = None,
                out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                w: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        _check(lib.ofb_moe_forward(ctypes.byref(self._cfg), ctypes.byref(self._w), _ptr(x),
                                   _ptr(resid), _ptr(out), T, _ptr(idx), _ptr(w), self.ws.handle,
                                   _stream(stream)))
        return out

    def forward_profiled(self, x: torch.Tensor, out: torch.Tensor, stream=None):
        """Runs one layer and returns the device ms of (routing, plan, up, down)."""
        ms = (ctypes.c_float * 4)()
        _check(lib.ofb_moe_forward_profiled(ctypes.byref(self._cfg), ctypes.byref(self._w), _ptr(x),
                                            None, _ptr(out), x.shape[0], self.ws.handle,
                                            _stream(stream), ms))
        return list(ms)

    def forward_noalloc(self, x: torch.Tensor, resid: torch.Tensor | None = None,
                        out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                        w: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """forward() through ofb_moe_forward_noalloc (fixed in-library scratch)."""
        if out is None:
            out = torch.empty_like(x)
        _check(lib.ofb_moe_forward_noalloc(ctypes.byref(self._cfg), ctypes.byref(self._w), _ptr(x),
                                           _ptr(resid), _ptr(out), x.shape[0], _ptr(idx), _ptr(w),
                                           _stream(stream)))
        return out

    def route(self, x: torch.Tensor, stream=None):
        T = x.shape[0]
        idx = torch.empty(T, self.shape.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.shape.top_k, dtype=torch.float32, device=x.device)
        _check(lib.ofb_route(ctypes.byref(self._cfg), _ptr(self.weights.router), _ptr(x), T,
                             _ptr(idx), _ptr(w), self.ws.handle, _stream(stream)))
        return idx, w
