"""Expert-parallel MoE layers over torch.distributed (one process per GPU).

Rank r of n owns the routed experts [r*E/n, (r+1)*E/n) of every layer (the
contiguous layout's expert range) and the tokens [r*T/n, (r+1)*T/n) of a step;
the router and the shared expert are replicated. One layer, on every rank:

  1. route own tokens (softmax / top-k over all E experts), ofb_route_certified;
  2. dispatch plan: slots grouped by destination rank, ofb_ep_plan, and the
     send buffers (x rows, {local expert, weight} pairs), ofb_ep_pack;
  3. all-to-all of the per-rank counts, then of rows and pairs;
  4. grouped expert SwiGLU on the received rows, out = w * y, ofb_moe_experts;
  5. all-to-all of the results back to the rows' owners;
  6. out = resid + g * shared(x) (ofb_moe_shared), then the routed terms
     added in top-k order (ofb_ep_combine).

The exchange is NCCL (or gloo, for host tests) through torch.distributed;
every computation is a kernel of libornith_cuda.so, reached through `EPOps`.
The reference runs its MoE block on one CPU (engine/src/model.c:992-1143); the
per-(token, expert) arithmetic is that block's, the decomposition over ranks
is this module's.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import torch
import torch.distributed as dist


def _binding():
    """The package's ofb.py, under the module name every loader of this
    (hyphenated, so not importable) directory uses."""
    name = "ornith_flight_b200.ofb"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                                         "ofb.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


ofb = _binding()


class EPOps:
    """Device implementation of the per-rank steps (C ABI of libornith_cuda.so)."""

    def __init__(self, shape: ofb.LayerShape, world: int, max_tokens: int):
        self.shape = shape
        self.world = world
        self.epr = shape.n_experts // world
        self.full_cfg = shape.config()
        self.loc_shape = ofb.LayerShape(shape.d_model, shape.hidden, self.epr, 1, ofb.LAYOUT_CONTIGUOUS,
                                        shape.routing, shape.renorm, shape.shared_gate)
        self.loc_cfg = self.loc_shape.config()
        # routing and the shared expert: a workspace of the full layer
        self.ws_full = ofb.Workspace(shape, max_tokens)
        # received rows: every token of every rank may route here
        self.max_rows = max(1, max_tokens * world * shape.top_k)
        self.ws_loc = ofb.Workspace(self.loc_shape, self.max_rows)

    def _struct(self, lw: ofb.LayerWeights):
        s = getattr(lw, "_ep_struct", None)
        if s is None:
            s = lw.struct()
            lw._ep_struct = s
        return s

    def route(self, lw: ofb.LayerWeights, x, idx, w):
        # the layer's certified routing: indices bit-exact, weights within 1e-5
        ofb._check(ofb.lib.ofb_route_certified(ctypes.byref(self.full_cfg), ofb._ptr(lw.router), ofb._ptr(x),
                                               x.shape[0], ofb._ptr(idx), ofb._ptr(w), self.ws_full.handle,
                                               ofb._stream()))

    def plan(self, idx, send_counts, slot_of, asg_of):
        T, K = idx.shape
        ofb._check(ofb.lib.ofb_ep_plan(ofb._ptr(idx), T, K, self.epr, self.world, ofb._ptr(send_counts),
                                       ofb._ptr(slot_of), ofb._ptr(asg_of), ofb._stream()))

    def pack(self, x, idx, w, asg_of, send_x, send_meta):
        T, K = idx.shape
        ofb._check(ofb.lib.ofb_ep_pack(ofb._ptr(x), ofb._ptr(idx), ofb._ptr(w), T, K, x.shape[1], self.epr,
                                       ofb._ptr(asg_of), ofb._ptr(send_x), ofb._ptr(send_meta), ofb._stream()))

    def experts(self, lw: ofb.LayerWeights, rows, meta, out):
        ofb._check(ofb.lib.ofb_moe_experts(ctypes.byref(self.loc_cfg), ctypes.byref(self._struct(lw)), ofb._ptr(rows),
                                           rows.shape[0], ofb._ptr(meta), ofb._ptr(out), self.ws_loc.handle,
                                           ofb._stream()))

    def shared(self, lw: ofb.LayerWeights, x, resid, out):
        ofb._check(ofb.lib.ofb_moe_shared(ctypes.byref(self.full_cfg), ctypes.byref(self._struct(lw)), ofb._ptr(x),
                                          ofb._ptr(resid), ofb._ptr(out), x.shape[0], self.ws_full.handle,
                                          ofb._stream()))

    def combine(self, y_back, slot_of, out):
        T, D = out.shape
        K = slot_of.shape[0] // max(T, 1)
        ofb._check(ofb.lib.ofb_ep_combine(ofb._ptr(y_back), ofb._ptr(slot_of), T, K, D, ofb._ptr(out),
                                          ofb._stream()))

    def rmsnorm(self, x, out, eps: float = 1e-6):
        ofb._check(ofb.lib.ofb_rmsnorm(ofb._ptr(x), x.shape[0], x.shape[1], eps, ofb._ptr(out), ofb._stream()))


class EPLayer:
    """One MoE layer whose routed experts are split over the ranks of `group`."""

    def __init__(self, shape: ofb.LayerShape, weights: ofb.LayerWeights, ops, max_tokens: int, device,
                 group=None):
        self.shape = shape
        self.weights = weights
        self.ops = ops
        self.group = group
        self.world = dist.get_world_size(group)
        if shape.n_experts % self.world:
            raise ValueError(f"{shape.n_experts} experts do not split over {self.world} ranks")
        if shape.layout != ofb.LAYOUT_CONTIGUOUS:
            raise ValueError("expert parallelism needs the contiguous layout")
        D, K = shape.d_model, shape.top_k
        TK = max_tokens * K
        rows = max_tokens * self.world * K
        i32, f32 = torch.int32, torch.float32
        self.idx = torch.empty(max_tokens, K, dtype=i32, device=device)
        self.w = torch.empty(max_tokens, K, dtype=f32, device=device)
        self.send_counts = torch.empty(self.world, dtype=i32, device=device)
        self.recv_counts = torch.empty(self.world, dtype=i32, device=device)
        self.slot_of = torch.empty(TK, dtype=i32, device=device)
        self.asg_of = torch.empty(TK, dtype=i32, device=device)
        self.send_x = torch.empty(TK, D, dtype=f32, device=device)
        self.send_meta = torch.empty(TK, 2, dtype=i32, device=device)
        self.recv_x = torch.empty(rows, D, dtype=f32, device=device)
        self.recv_meta = torch.empty(rows, 2, dtype=i32, device=device)
        self.y_rows = torch.empty(rows, D, dtype=f32, device=device)
        self.y_back = torch.empty(TK, D, dtype=f32, device=device)
        self.last_counts = None

    def forward(self, x: torch.Tensor, resid: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
        """out = resid + g*shared(x) + sum_k w_k * expert_k(x) for this rank's tokens x."""
        T = x.shape[0]
        K = self.shape.top_k
        TK = T * K
        idx, w = self.idx[:T], self.w[:T]
        ops, g = self.ops, self.group
        ops.route(self.weights, x, idx, w)
        ops.plan(idx, self.send_counts, self.slot_of[:TK], self.asg_of[:TK])
        ops.pack(x, idx, w, self.asg_of[:TK], self.send_x[:TK], self.send_meta[:TK])
        dist.all_to_all_single(self.recv_counts, self.send_counts, group=g)
        counts = torch.stack([self.send_counts, self.recv_counts]).cpu()  # the one host sync per layer
        sc, rc = counts[0].tolist(), counts[1].tolist()
        R = sum(rc)
        self.last_counts = (sc, rc)
        dist.all_to_all_single(self.recv_x[:R], self.send_x[:TK], rc, sc, group=g)
        dist.all_to_all_single(self.recv_meta[:R], self.send_meta[:TK], rc, sc, group=g)
        if R:
            ops.experts(self.weights, self.recv_x[:R], self.recv_meta[:R], self.y_rows[:R])
        dist.all_to_all_single(self.y_back[:TK], self.y_rows[:R], sc, rc, group=g)
        ops.shared(self.weights, x, resid, out)
        ops.combine(self.y_back[:TK], self.slot_of[:TK], out)
        return out


class EPGroup:
    """Device-side exchange over NVLink for the ranks of `group`
    (ofb_ep_group_*: every rank maps every other rank's window; rows, results
    and epoch-tagged flags travel as peer stores, no host synchronisation).
    Set-up gathers the ranks' IPC handles with torch.distributed."""

    def __init__(self, shape: ofb.LayerShape, max_tokens: int, device, group=None):
        self.shape = shape
        self.max_tokens = max_tokens
        self._cfg = shape.config()
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        hb = ofb.lib  # noqa: F841 (binding loaded)
        h = (ctypes.c_uint8 * 64)()
        self.handle = ctypes.c_void_p()
        ofb._check(ofb.lib.ofb_ep_group_create(ctypes.byref(self._cfg), rank, world, max_tokens,
                                               ctypes.byref(self.handle), h))
        mine = torch.tensor(list(h), dtype=torch.uint8, device=device)
        every = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        allh = (ctypes.c_uint8 * (world * 64))(*every.cpu().tolist())
        ofb._check(ofb.lib.ofb_ep_group_connect(self.handle, allh))

    def forward(self, weights: ofb.LayerWeights, wstruct, x, resid, out):
        ofb._check(ofb.lib.ofb_ep_layer_forward(self.handle, ctypes.byref(wstruct), ofb._ptr(x), ofb._ptr(resid),
                                                ofb._ptr(out), x.shape[0], ofb._stream()))
        return out

    def device_errors(self) -> int:
        b = ctypes.c_uint()
        ofb._check(ofb.lib.ofb_ep_group_device_errors(self.handle, ctypes.byref(b)))
        return b.value

    def close(self):
        if self.handle:
            ofb._check(ofb.lib.ofb_ep_group_destroy(self.handle))
            self.handle = None


class EPLayerP2P:
    """One expert-parallel MoE layer through an EPGroup (one C call per layer):
    weights = the full router, shared expert and gate vector plus this rank's
    routed experts (ofb.make_layer_slice)."""

    def __init__(self, shape: ofb.LayerShape, weights: ofb.LayerWeights, group: EPGroup):
        self.shape = shape
        self.weights = weights
        self.group = group
        self._w = weights.struct()

    def forward(self, x: torch.Tensor, resid: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
        return self.group.forward(self.weights, self._w, x, resid, out)


class LocalLayer:
    """One rank holding every expert: the whole layer, no exchange."""

    def __init__(self, shape: ofb.LayerShape, weights: ofb.LayerWeights, max_tokens: int):
        self.shape = shape
        self.layer = ofb.MoeLayer(shape, weights, max_tokens)

    def forward(self, x: torch.Tensor, resid: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
        return self.layer.forward(x, resid, out=out)


class EPStack:
    """A stack of expert-parallel MoE layers: x <- x + MoE_l(rmsnorm(x)) for
    each layer l (the FFN half of the model's blocks, engine/src/model.c:992,
    with unit norm weights and no attention)."""

    def __init__(self, layers: list, ops, max_tokens: int, device):
        self.layers = layers
        self.ops = ops  # EPOps, or None: the library's RMSNorm directly
        D = layers[0].shape.d_model
        self.xn = torch.empty(max_tokens, D, dtype=torch.float32, device=device)
        self.bufs = torch.empty(2, max_tokens, D, dtype=torch.float32, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Runs every layer over this rank's tokens x (left unchanged); returns
        the final residual stream (a view of an internal buffer)."""
        T = x.shape[0]
        xn, cur = self.xn[:T], x
        for i, layer in enumerate(self.layers):
            nxt = self.bufs[i % 2, :T]
            if self.ops is not None:
                self.ops.rmsnorm(cur, xn)
            else:
                ofb._check(ofb.lib.ofb_rmsnorm(ofb._ptr(cur), T, cur.shape[1], 1e-6, ofb._ptr(xn), ofb._stream()))
            layer.forward(xn, cur, nxt)
            cur = nxt
        return cur
