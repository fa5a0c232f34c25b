"""ctypes binding of the CPU oracle (liboracle.so) and of the reference's own
compiled dequant (oracle/_ref/libref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference legs as the checker, never by the product.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref.so")

TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 12, 14
LAYOUT_CONTIGUOUS, LAYOUT_INTERLEAVED = 0, 1
ROUTE_FORWARD, ROUTE_GET_ROUTING = 0, 1


class OrcCfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "d_model", "hidden", "n_experts", "top_k", "layout", "routing", "renorm", "shared_gate")]


class OrcWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
        "shexp_gate_v")]


def _np_ptr(a):
    return None if a is None else a.ctypes.data


def load_oracle():
    if not os.path.exists(ORACLE_PATH):
        raise ImportError(f"{ORACLE_PATH} missing: run `make -C {HERE}`")
    L = ctypes.CDLL(ORACLE_PATH)
    vp, u64, i32, f32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_float
    L.orc_fp16_to_fp32.restype, L.orc_fp16_to_fp32.argtypes = f32, [ctypes.c_uint16]
    L.orc_dequant_tensor.restype, L.orc_dequant_tensor.argtypes = i32, [vp, i32, u64, vp]
    L.orc_dequant_slice.restype, L.orc_dequant_slice.argtypes = i32, [vp, i32, u64, u64, i32, vp]
    L.orc_expf.restype, L.orc_expf.argtypes = f32, [f32]
    L.orc_moe_forward.restype = i32
    L.orc_moe_forward.argtypes = [ctypes.POINTER(OrcCfg), ctypes.POINTER(OrcWeights), vp, vp, i32,
                                  vp, vp, vp]
    L.orc_matmul.restype, L.orc_matmul.argtypes = None, [vp, vp, vp, i32, i32, i32]
    L.orc_expf_batch.restype, L.orc_expf_batch.argtypes = None, [vp, vp, u64]
    L.orc_synth_blocks.restype, L.orc_synth_blocks.argtypes = None, [vp, i32, u64, u64, u64, u64]
    L.orc_synth_normal.restype, L.orc_synth_normal.argtypes = None, [vp, u64, u64, u64, f32]
    return L


def load_ref():
    """The reference's own engine/src/gguf.c, or None if it was not built."""
    if not os.path.exists(REF_PATH):
        return None
    L = ctypes.CDLL(REF_PATH)
    vp, u64, i32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
    L.ref_dequant_tensor.restype, L.ref_dequant_tensor.argtypes = i32, [vp, i32, u64, vp]
    L.ref_dequant_slice.restype, L.ref_dequant_slice.argtypes = i32, [vp, i32, u64, u64, i32, vp]
    return L


_orc = None


def orc():
    global _orc
    if _orc is None:
        _orc = load_oracle()
    return _orc


def dequant(blocks: np.ndarray, qtype: int, n_elems: int, lib=None) -> np.ndarray:
    out = np.empty(n_elems, dtype=np.float32)
    L = lib or orc()
    fn = L.orc_dequant_tensor if hasattr(L, "orc_dequant_tensor") else L.ref_dequant_tensor
    assert fn(_np_ptr(np.ascontiguousarray(blocks)), qtype, n_elems, _np_ptr(out)) == 1
    return out


def dequant_slice(blocks: np.ndarray, qtype: int, n_elems: int, n_experts: int, expert: int,
                  lib=None) -> np.ndarray:
    out = np.empty(n_elems // n_experts, dtype=np.float32)
    L = lib or orc()
    fn = L.orc_dequant_slice if hasattr(L, "orc_dequant_slice") else L.ref_dequant_slice
    assert fn(_np_ptr(np.ascontiguousarray(blocks)), qtype, n_elems, n_experts, expert,
              _np_ptr(out)) == 1
    return out


def expf_batch(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    orc().orc_expf_batch(_np_ptr(x), _np_ptr(out), x.size)
    return out


def moe_forward(cfg: dict, w: dict, x: np.ndarray, resid: np.ndarray | None = None):
    """CPU MoE layer. cfg: d_model, hidden, n_experts, top_k, layout, routing,
    renorm, shared_gate. w: numpy arrays router, gate_exps, up_exps, down_exps,
    gate_shexp, up_shexp, down_shexp, shexp_gate (any may be None)."""
    c = OrcCfg(*(int(cfg[k]) for k in ("d_model", "hidden", "n_experts", "top_k", "layout",
                                         "routing", "renorm", "shared_gate")))
    keep = {k: (None if v is None else np.ascontiguousarray(v)) for k, v in w.items()}
    ww = OrcWeights(*(_np_ptr(keep.get(k)) for k in (
        "router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
        "shexp_gate")))
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.shape[0]
    out = np.empty_like(x)
    idx = np.empty((T, c.top_k), dtype=np.uint32)
    wt = np.empty((T, c.top_k), dtype=np.float32)
    r = None if resid is None else np.ascontiguousarray(resid, dtype=np.float32)
    ok = orc().orc_moe_forward(ctypes.byref(c), ctypes.byref(ww), _np_ptr(x), _np_ptr(r), T,
                               _np_ptr(out), _np_ptr(idx), _np_ptr(wt))
    assert ok == 1, "oracle rejected the arguments"
    return out, idx, wt


_ref_keepalive = None


def use_reference_dequant(enable: bool = True) -> bool:
    """Make the oracle layer call the reference's own compiled dequant
    (oracle/_ref/libref.so) instead of the restatement. Returns False when the
    reference build is absent."""
    global _ref_keepalive
    L = orc()
    L.orc_set_dequant.restype = None
    L.orc_set_dequant.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    if not enable:
        L.orc_set_dequant(None, None)
        return True
    ref = load_ref()
    if ref is None:
        return False
    _ref_keepalive = ref
    t = ctypes.cast(ref.ref_dequant_tensor, ctypes.c_void_p).value
    s = ctypes.cast(ref.ref_dequant_slice, ctypes.c_void_p).value
    L.orc_set_dequant(t, s)
    return True


# ---- seeded synthetic layers, built on the host without the product library ----
# Stream ids and distributions of the library's make_layer / make_tokens.
STREAM_GATE, STREAM_UP, STREAM_DOWN, STREAM_GATE_SH, STREAM_UP_SH, STREAM_DOWN_SH = 1, 2, 3, 4, 5, 6
STREAM_ROUTER, STREAM_GATE_V, STREAM_X = 7, 8, 9
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210}


def synth_blocks(qtype: int, n_blocks: int, seed: int, stream_id: int, first_block: int = 0) -> np.ndarray:
    out = np.empty(n_blocks * BLOCK_BYTES[qtype], dtype=np.uint8)
    orc().orc_synth_blocks(_np_ptr(out), qtype, n_blocks, first_block, seed, stream_id)
    return out


def synth_normal(n: int, seed: int, stream_id: int, sigma: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    orc().orc_synth_normal(_np_ptr(out), n, seed, stream_id, sigma)
    return out


def make_layer_host(d_model=2048, hidden=512, n_experts=256, layout=LAYOUT_CONTIGUOUS, seed=0,
                    shared=True, router_bias=None) -> dict:
    """The bytes of the library's make_layer(shape, seed) as numpy arrays
    (router laid out per `layout`: [E][D] contiguous, [D][E] interleaved)."""
    nb = hidden * d_model // 256
    E, D = n_experts, d_model
    r = synth_normal(E * D, seed, STREAM_ROUTER, 0.02).reshape(E, D)
    if router_bias is not None:
        r[:, 0] = np.asarray(router_bias, dtype=np.float32)
    if layout == LAYOUT_INTERLEAVED:
        r = np.ascontiguousarray(r.T)
    w = dict(router=r.reshape(-1),
             gate_exps=synth_blocks(TYPE_Q4_K, E * nb, seed, STREAM_GATE),
             up_exps=synth_blocks(TYPE_Q4_K, E * nb, seed, STREAM_UP),
             down_exps=synth_blocks(TYPE_Q6_K, E * nb, seed, STREAM_DOWN),
             gate_shexp=None, up_shexp=None, down_shexp=None, shexp_gate=None)
    if shared:
        w.update(gate_shexp=synth_blocks(TYPE_Q4_K, nb, seed, STREAM_GATE_SH),
                 up_shexp=synth_blocks(TYPE_Q4_K, nb, seed, STREAM_UP_SH),
                 down_shexp=synth_blocks(TYPE_Q6_K, nb, seed, STREAM_DOWN_SH),
                 shexp_gate=synth_normal(D, seed, STREAM_GATE_V, 0.02))
    return w


def make_tokens_host(d_model: int, n_tokens: int, seed: int) -> np.ndarray:
    return synth_normal(n_tokens * d_model, seed, STREAM_X, 1.0).reshape(n_tokens, d_model)


def _chunk_worker(args):
    cfg, seed, bias, x = args
    w = make_layer_host(cfg["d_model"], cfg["hidden"], cfg["n_experts"], cfg["layout"], seed,
                        router_bias=bias)
    return moe_forward(cfg, w, x)


def moe_forward_seeded_parallel(cfg: dict, seed: int, x: np.ndarray, router_bias=None, procs=None,
                                chunk=128):
    """moe_forward over the seeded synthetic layer make_layer_host(seed) for
    many tokens, split into token chunks run by a pool of processes (each
    builds the layer itself). The layer is per token, so the result equals
    one call over all tokens."""
    import multiprocessing as mp
    procs = procs or min(32, os.cpu_count() or 1)
    jobs = [(cfg, seed, router_bias, x[i:i + chunk]) for i in range(0, x.shape[0], chunk)]
    with mp.get_context("spawn").Pool(min(procs, len(jobs))) as pool:
        res = pool.map(_chunk_worker, jobs)
    return (np.concatenate([r[0] for r in res]), np.concatenate([r[1] for r in res]),
            np.concatenate([r[2] for r in res]))
