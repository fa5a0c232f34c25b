"""Expert-parallel check on N GPUs (run by tests/test_gpu_ep.py under torchrun).

Every rank holds experts [r*E/N, (r+1)*E/N) and tokens [r*T/N, ...) of seeded
layers; the expert-parallel result must match the single-GPU layer
(ofb_moe_forward of the whole layer on the same rank) on the rank's tokens,
one layer and a 3-layer stack, at a decode-sized and a tensor-core-sized
batch. Rank 0 also checks a few tokens against the oracle."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from conftest import load_ep, load_ofb  # noqa: E402
from test_gpu_moe import TOL, TOL_BF16, oracle_layer, rel_err  # noqa: E402


def nccl_comm(rank, world, dev):
    """A raw ncclComm_t from the NCCL library torch loaded (the unique id is
    broadcast with torch.distributed), for ofb_ep_group_create_nccl."""
    import ctypes

    class UID(ctypes.Structure):
        _fields_ = [("internal", ctypes.c_ubyte * 128)]

    nccl = ctypes.CDLL("libnccl.so.2")
    uid = UID()
    if rank == 0:
        assert nccl.ncclGetUniqueId(ctypes.byref(uid)) == 0
    t = torch.tensor(list(uid.internal) if rank == 0 else [0] * 128, dtype=torch.uint8, device=dev)
    dist.broadcast(t, 0)
    uid = UID((ctypes.c_ubyte * 128)(*t.cpu().tolist()))
    comm = ctypes.c_void_p()
    rc = nccl.ncclCommInitRank(ctypes.byref(comm), world, uid, rank)
    assert rc == 0, f"ncclCommInitRank: {rc}"
    return nccl, comm


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=dev)
    ofb, ep = load_ofb(), load_ep()
    # hidden 768: every part runs the fp32 decode kernels (tensor-core kernels
    # need hidden <= 512), so the 3-layer stacks compare at 1e-3 with no
    # routing flips; hidden 256 at 40 tokens per rank: the bf16 tensor-core
    # kernels
    shapes = {4 * world: ofb.LayerShape(d_model=512, hidden=768, n_experts=16, top_k=4),
              40 * world: ofb.LayerShape(d_model=512, hidden=256, n_experts=16, top_k=4)}
    fails = []
    for T_global, shape in shapes.items():
        epr = shape.n_experts // world
        tpr = T_global // world
        ops = ep.EPOps(shape, world, max_tokens=tpr)
        seeds = [31 + l for l in range(3)]
        layers = [ep.EPLayer(shape, ofb.make_layer_slice(shape, s, rank * epr, (rank + 1) * epr, device=dev), ops, tpr,
                             dev) for s in seeds]
        x_all = ofb.make_tokens(shape, T_global, seed=5).to(dev)
        x = x_all[rank * tpr:(rank + 1) * tpr].contiguous()
        # single-GPU reference on this rank: the whole layers, all tokens
        full = [ofb.MoeLayer(shape, ofb.make_layer(shape, s, device=dev), T_global) for s in seeds]
        tol = TOL if ofb.decode_path(tpr * shape.top_k * world, shape.hidden) and ofb.decode_path(T_global, shape.hidden) else TOL_BF16
        out = torch.empty_like(x)
        layers[0].forward(x, x, out)
        ref = full[0].forward(x_all, x_all)[rank * tpr:(rank + 1) * tpr]
        e1 = rel_err((out - x).cpu().numpy(), (ref - x).cpu().numpy())
        got = ep.EPStack(layers, ops, tpr, dev).forward(x)
        cur = x_all.clone()
        for f in full:
            xn = torch.empty_like(cur)
            ops.rmsnorm(cur, xn)
            cur = f.forward(xn, cur)
        e2 = rel_err(got.cpu().numpy(), cur[rank * tpr:(rank + 1) * tpr].cpu().numpy())
        if rank == 0:
            want, _, _ = oracle_layer(__import__("binding"), shape, ofb.make_layer(shape, seeds[0], device="cpu"),
                                      x[:3].cpu().numpy(), x[:3].cpu().numpy())
            e3 = rel_err((out[:3] - x[:3]).cpu().numpy(), want - x[:3].cpu().numpy())
        else:
            e3 = 0.0
        print(f"rank {rank} T={T_global}: layer {e1:.2e} stack {e2:.2e} oracle {e3:.2e} (tol {tol})", flush=True)
        if not (e1 <= tol and e2 <= tol and e3 <= tol):
            fails.append(T_global)
        # the device-side exchange (EPGroup / EPLayerP2P): same layers, same checks
        grp = ep.EPGroup(shape, tpr, dev)
        p2p = [ep.EPLayerP2P(shape, l.weights, grp) for l in layers]
        out2 = torch.empty_like(x)
        p2p[0].forward(x, x, out2)
        e4 = rel_err((out2 - x).cpu().numpy(), (ref - x).cpu().numpy())
        got2 = ep.EPStack(p2p, None, tpr, dev).forward(x)
        e5 = rel_err(got2.cpu().numpy(), cur[rank * tpr:(rank + 1) * tpr].cpu().numpy())
        # repeated layers in one stream: the epochs advance, results repeat
        again = ep.EPStack(p2p, None, tpr, dev).forward(x)
        e6 = rel_err(again.cpu().numpy(), got2.cpu().numpy())
        errs = grp.device_errors()
        grp.close()
        # the same layer through a group made from a raw NCCL communicator
        import ctypes
        nccl, comm = nccl_comm(rank, world, dev)
        h = ctypes.c_void_p()
        ofb._check(ofb.lib.ofb_ep_group_create_nccl(ctypes.byref(shape.config()), comm, tpr, ctypes.byref(h),
                                                    ofb._stream()))
        out3 = torch.empty_like(x)
        ofb._check(ofb.lib.ofb_ep_layer_forward(h, ctypes.byref(layers[0].weights.struct()), ofb._ptr(x),
                                                ofb._ptr(x), ofb._ptr(out3), tpr, ofb._stream()))
        torch.cuda.synchronize()
        e7 = rel_err(out3.cpu().numpy(), out2.cpu().numpy())
        ofb._check(ofb.lib.ofb_ep_group_destroy(h))
        nccl.ncclCommDestroy(comm)
        print(f"rank {rank} T={T_global} nccl-made group: vs p2p {e7:.2e}", flush=True)
        if not e7 <= 1e-6:
            fails.append(-2 * T_global)
        print(f"rank {rank} T={T_global} p2p: layer {e4:.2e} stack {e5:.2e} repeat {e6:.2e} device errors {errs}",
              flush=True)
        if not (e4 <= tol and e5 <= tol and e6 <= 1e-6 and errs == 0):
            fails.append(-T_global)
    ok = torch.tensor([0 if fails else 1], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0 and ok.item() == 1:
        print("ep_multi_gpu: ok", flush=True)
    sys.exit(0 if ok.item() == 1 else 1)


if __name__ == "__main__":
    main()
