"""Expert-parallel host logic on the CPU: world_size-2 gloo process groups run
EPLayer / EPStack (ornith-flight_b200/ep.py) with the oracle as each rank's
compute, and must reproduce the single-process oracle layer exactly.

OracleOps restates, in numpy, the index semantics of the device steps
(ofb_ep_plan: slots grouped by destination rank, assignment order kept inside
a rank; ofb_ep_pack; ofb_ep_combine: routed terms summed in top-k order, then
added) and computes the experts with the oracle (oracle/moe.c). The test
checks the exchange protocol: count exchange, variable all-to-all splits,
the return trip and the combine indexing."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_ep, load_ofb

SHAPE = dict(d_model=256, hidden=256, n_experts=8, top_k=2)
T_GLOBAL = 6
SEED = 11


class OracleOps:
    """Per-rank steps of an expert-parallel layer on CPU tensors (test only)."""

    def __init__(self, binding, shape, world):
        self.b = binding
        self.shape = shape
        self.epr = shape.n_experts // world
        self.nb = shape.q4k_blocks_per_expert
        self.cfg = dict(d_model=shape.d_model, hidden=shape.hidden, n_experts=shape.n_experts,
                        top_k=shape.top_k, layout=0, routing=shape.routing, renorm=shape.renorm,
                        shared_gate=shape.shared_gate)
        lib = binding.orc()
        lib.orc_route_token.argtypes = [ctypes.POINTER(binding.OrcCfg)] + [ctypes.c_void_p] * 4
        lib.orc_route_token.restype = None
        self.lib = lib

    def route(self, lw, x, idx, w):
        c = self.b.OrcCfg(*(int(self.cfg[k]) for k in ("d_model", "hidden", "n_experts", "top_k", "layout",
                                                         "routing", "renorm", "shared_gate")))
        xn = np.ascontiguousarray(x.numpy())
        r = np.ascontiguousarray(lw.router.numpy())
        ii = np.empty((x.shape[0], self.shape.top_k), np.uint32)
        ww = np.empty((x.shape[0], self.shape.top_k), np.float32)
        for t in range(x.shape[0]):
            self.lib.orc_route_token(ctypes.byref(c), xn[t].ctypes.data, r.ctypes.data, ii[t].ctypes.data,
                                     ww[t].ctypes.data)
        idx.copy_(torch.from_numpy(ii.view(np.int32)))
        w.copy_(torch.from_numpy(ww))

    def plan(self, idx, send_counts, slot_of, asg_of):
        dest = (idx.reshape(-1).numpy().astype(np.int64) // self.epr)
        order = np.argsort(dest, kind="stable")
        asg_of.copy_(torch.from_numpy(order.astype(np.int32)))
        slots = np.empty_like(order)
        slots[order] = np.arange(order.size)
        slot_of.copy_(torch.from_numpy(slots.astype(np.int32)))
        send_counts.copy_(torch.from_numpy(np.bincount(dest, minlength=send_counts.numel()).astype(np.int32)))

    def pack(self, x, idx, w, asg_of, send_x, send_meta):
        K = idx.shape[1]
        a = asg_of.numpy()
        e = idx.reshape(-1).numpy()[a]
        send_x.copy_(x[torch.from_numpy(a // K)])
        meta = np.stack([e % self.epr, w.reshape(-1).numpy()[a].view(np.int32)], axis=1)
        send_meta.copy_(torch.from_numpy(meta.astype(np.int32)))

    def _one_expert(self, lw, e):
        q4, q6 = self.nb * 144, self.nb * 210
        return dict(router=None, gate_exps=lw.gate_exps.numpy()[e * q4:(e + 1) * q4],
                    up_exps=lw.up_exps.numpy()[e * q4:(e + 1) * q4],
                    down_exps=lw.down_exps.numpy()[e * q6:(e + 1) * q6],
                    gate_shexp=None, up_shexp=None, down_shexp=None, shexp_gate=None)

    def experts(self, lw, rows, meta, out):
        cfg1 = dict(self.cfg, n_experts=1, top_k=1, shared_gate=0)
        m = meta.numpy()
        for r in range(rows.shape[0]):
            e, wt = int(m[r, 0]), m[r, 1:2].view(np.float32)[0]
            if wt < np.float32(1e-6):  # model.c:1066 skip rule
                out[r] = 0.0
                continue
            y, _, _ = self.b.moe_forward(cfg1, self._one_expert(lw, e), rows[r:r + 1].numpy())
            out[r] = torch.from_numpy(wt * y[0])

    def shared(self, lw, x, resid, out):
        # a one-expert layer whose routed expert is all-zero blocks: out = resid + g*shared(x)
        cfg1 = dict(self.cfg, n_experts=1, top_k=1)
        z4, z6 = np.zeros(self.nb * 144, np.uint8), np.zeros(self.nb * 210, np.uint8)
        wd = dict(router=None, gate_exps=z4, up_exps=z4, down_exps=z6, gate_shexp=lw.gate_shexp.numpy(),
                  up_shexp=lw.up_shexp.numpy(), down_shexp=lw.down_shexp.numpy(), shexp_gate=lw.shexp_gate.numpy())
        o, _, _ = self.b.moe_forward(cfg1, wd, x.numpy(), None if resid is None else resid.numpy())
        out.copy_(torch.from_numpy(o))

    def combine(self, y_back, slot_of, out):
        T = out.shape[0]
        K = slot_of.numel() // T
        y, s = y_back.numpy(), slot_of.numpy()
        o = out.numpy().copy()
        for t in range(T):
            r = np.zeros(out.shape[1], np.float32)
            for k in range(K):
                r = r + y[s[t * K + k]]
            o[t] = o[t] + r
        out.copy_(torch.from_numpy(o))

    def rmsnorm(self, x, out, eps=1e-6):
        xn = x.numpy()
        ss = (xn * xn).sum(axis=1, dtype=np.float32)
        inv = np.float32(1.0) / np.sqrt(ss / np.float32(xn.shape[1]) + np.float32(eps))
        out.copy_(torch.from_numpy((xn * inv[:, None]).astype(np.float32)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_layers, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import binding
        ofb = load_ofb()
        ep = load_ep()
        shape = ofb.LayerShape(**SHAPE)
        epr = shape.n_experts // world
        ops = OracleOps(binding, shape, world)
        tpr = T_GLOBAL // world
        layers = [ep.EPLayer(shape, ofb.make_layer_slice(shape, SEED + l, rank * epr, (rank + 1) * epr, device="cpu"),
                             ops, tpr, "cpu") for l in range(n_layers)]
        x = ofb.make_tokens(shape, T_GLOBAL, seed=SEED)[rank * tpr:(rank + 1) * tpr].contiguous()
        if n_layers == 1:
            out = torch.empty_like(x)
            layers[0].forward(x, x, out)
        else:
            out = ep.EPStack(layers, ops, tpr, "cpu").forward(x).clone()
        q.put((rank, out.numpy(), layers[0].last_counts))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surfaces in the parent instead of hanging it
        q.put((rank, repr(e), None))


def _run(n_layers, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_layers, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out, counts = q.get(timeout=300)
        res[rank] = (out, counts)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r][0], str), f"rank {r} failed: {res[r][0]}"
    return np.concatenate([res[r][0] for r in range(world)]), [res[r][1] for r in range(world)]


def _oracle_layer(oracle, ofb, shape, seed, x, resid):
    lw = ofb.make_layer(shape, seed, device="cpu")
    cfg = dict(d_model=shape.d_model, hidden=shape.hidden, n_experts=shape.n_experts, top_k=shape.top_k,
               layout=0, routing=shape.routing, renorm=shape.renorm, shared_gate=shape.shared_gate)
    w = {k: (None if v is None else v.numpy()) for k, v in vars(lw).items() if not k.startswith("_")}
    w["shexp_gate"] = lw.shexp_gate.numpy()
    out, _, _ = oracle.moe_forward(cfg, w, x, resid)
    return out


def test_ep_layer_two_ranks_matches_oracle(ofb, oracle):
    shape = ofb.LayerShape(**SHAPE)
    x = ofb.make_tokens(shape, T_GLOBAL, seed=SEED).numpy()
    ref = _oracle_layer(oracle, ofb, shape, SEED, x, x)
    got, counts = _run(1)
    np.testing.assert_array_equal(got, ref)
    # the count exchange is consistent: what r sends to s, s receives from r
    (sc0, rc0), (sc1, rc1) = counts
    assert sc0[1] == rc1[0] and sc1[0] == rc0[1]
    assert sum(sc0) == sum(sc1) == (T_GLOBAL // 2) * shape.top_k


def test_ep_stack_two_ranks_matches_oracle(ofb, oracle):
    shape = ofb.LayerShape(**SHAPE)
    ops = OracleOps(oracle, shape, 1)
    cur = ofb.make_tokens(shape, T_GLOBAL, seed=SEED)
    for l in range(2):
        xn = torch.empty_like(cur)
        ops.rmsnorm(cur, xn)
        cur = torch.from_numpy(_oracle_layer(oracle, ofb, shape, SEED + l, xn.numpy(), cur.numpy()))
    got, _ = _run(2)
    np.testing.assert_array_equal(got, cur.numpy())


def test_ep_plan_semantics(ofb, oracle):
    """The numpy plan restated here: grouping by rank, stable inside a rank."""
    ops = OracleOps(oracle, ofb.LayerShape(**SHAPE), 4)
    idx = torch.tensor([[7, 0], [2, 3], [6, 1], [4, 5]], dtype=torch.int32)
    sc, so, ao = (torch.empty(4, dtype=torch.int32), torch.empty(8, dtype=torch.int32),
                  torch.empty(8, dtype=torch.int32))
    ops.plan(idx, sc, so, ao)
    assert sc.tolist() == [2, 2, 2, 2]
    assert ao.tolist() == [1, 5, 2, 3, 6, 7, 0, 4]
    assert all(so[a] == s for s, a in enumerate(ao.tolist()))
