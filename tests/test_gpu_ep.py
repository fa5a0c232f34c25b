"""Expert-parallel building blocks on the GPU through the C ABI: the dispatch
plan / pack / combine kernels against their numpy restatement, the grouped
expert entry (ofb_moe_experts) and the shared-expert entry (ofb_moe_shared)
against the oracle, and the whole EPLayer at one rank (NCCL) and at two
(torchrun child, when two GPUs are visible).

Tolerances as the layer tests: per row, max|gpu - ref| <= 1e-3 * max|ref| on
the fp32 decode path (<= 32 rows), 2e-2 on the bf16 tensor-core path."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist

from conftest import ROOT, load_ep
from test_ep_gloo import OracleOps
from test_gpu_moe import TOL, TOL_BF16, oracle_layer, rel_err

pytestmark = pytest.mark.gpu
SMALL = dict(d_model=512, hidden=256, n_experts=16, top_k=4)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,T", [(2, 7), (4, 33), (8, 300)])
def test_ep_plan_pack_combine(ofb, oracle, cuda, world, T):
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=64, top_k=8)
    ep = load_ep()
    ops = ep.EPOps.__new__(ep.EPOps)  # kernels only: no workspaces needed
    ops.world, ops.epr = world, shape.n_experts // world
    ref = OracleOps(oracle, shape, world)
    g = torch.Generator().manual_seed(T)
    idx = torch.stack([torch.randperm(shape.n_experts, generator=g)[:shape.top_k] for _ in range(T)]).int()
    w = torch.rand(T, shape.top_k, generator=g)
    x = torch.randn(T, shape.d_model, generator=g)
    TK = T * shape.top_k
    outs = {}
    for name, o, dev in (("gpu", ops, cuda), ("ref", ref, "cpu")):
        sc = torch.empty(world, dtype=torch.int32, device=dev)
        so = torch.empty(TK, dtype=torch.int32, device=dev)
        ao = torch.empty(TK, dtype=torch.int32, device=dev)
        o.plan(idx.to(dev), sc, so, ao)
        sx = torch.empty(TK, shape.d_model, device=dev)
        sm = torch.empty(TK, 2, dtype=torch.int32, device=dev)
        o.pack(x.to(dev), idx.to(dev), w.to(dev), ao, sx, sm)
        y = torch.randn(TK, shape.d_model, generator=torch.Generator().manual_seed(5)).to(dev)
        out = x.to(dev).clone()
        o.combine(y, so, out)
        outs[name] = [t.cpu() for t in (sc, so, ao, sx, sm, out)]
    for a, b in zip(outs["gpu"], outs["ref"]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("R", [1, 6, 32, 90])
def test_moe_experts_matches_oracle(ofb, oracle, cuda, R):
    shape = ofb.LayerShape(**SMALL)
    ep = load_ep()
    world, rank = 2, 1
    epr = shape.n_experts // world
    lw = ofb.make_layer_slice(shape, 21, rank * epr, (rank + 1) * epr, device=cuda)
    ops = ep.EPOps(shape, world, max_tokens=max(1, R // shape.top_k + 1))
    g = torch.Generator().manual_seed(R)
    rows = ofb.make_tokens(shape, R, seed=R + 3)
    meta = torch.stack([torch.randint(0, epr, (R,), generator=g).int(),
                        torch.rand(R, generator=g).view(torch.int32)], dim=1).contiguous()
    meta[0, 1] = torch.tensor([5e-7], dtype=torch.float32).view(torch.int32)  # below the skip threshold
    out = torch.empty(R, shape.d_model, device=cuda)
    ops.experts(lw, rows.to(cuda), meta.to(cuda), out)
    want = torch.empty(R, shape.d_model)
    OracleOps(oracle, shape, world).experts(lw.to("cpu"), rows, meta, want)
    got = out.cpu().numpy()
    assert np.all(got[0] == 0.0)
    err = rel_err(got[1:], want.numpy()[1:]) if R > 1 else 0.0
    assert err <= (TOL if ofb.decode_path(R, 256) else TOL_BF16), f"relative error {err}"


@pytest.mark.parametrize("T", [3, 40])
def test_moe_shared_matches_oracle(ofb, oracle, cuda, T):
    shape = ofb.LayerShape(**SMALL)
    ep = load_ep()
    lw = ofb.make_layer_slice(shape, 22, 0, shape.n_experts, device=cuda)
    ops = ep.EPOps(shape, 1, max_tokens=T)
    x = ofb.make_tokens(shape, T, seed=T)
    r = ofb.make_tokens(shape, T, seed=T + 1)
    out = torch.empty(T, shape.d_model, device=cuda)
    ops.shared(lw, x.to(cuda), r.to(cuda), out)
    want = torch.empty(T, shape.d_model)
    OracleOps(oracle, shape, 1).shared(lw.to("cpu"), x, r, want)
    err = rel_err(out.cpu().numpy() - r.numpy(), want.numpy() - r.numpy())
    assert err <= (TOL if ofb.decode_path(T, 256) else TOL_BF16), f"relative error {err}"


@pytest.mark.parametrize("T", [8, 48])
def test_ep_layer_one_rank_matches_oracle(ofb, oracle, cuda, T):
    shape = ofb.LayerShape(**SMALL)
    ep = load_ep()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0, world_size=1,
                            device_id=cuda)
    try:
        lw = ofb.make_layer_slice(shape, 23, 0, shape.n_experts, device=cuda)
        ops = ep.EPOps(shape, 1, max_tokens=T)
        layer = ep.EPLayer(shape, lw, ops, T, cuda)
        x = ofb.make_tokens(shape, T, seed=7).to(cuda)
        out = torch.empty_like(x)
        layer.forward(x, x, out)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    full = ofb.make_layer(shape, 23, device="cpu")
    want, _, _ = oracle_layer(oracle, shape, full, x.cpu().numpy(), x.cpu().numpy())
    # routed rows = T * top_k: 32 rows stay on the fp32 path, 192 use the tensor cores
    err = rel_err(out.cpu().numpy() - x.cpu().numpy(), want - x.cpu().numpy())
    assert err <= (TOL if ofb.decode_path(T * shape.top_k, shape.hidden) else TOL_BF16), f"relative error {err}"


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus():
    port = _port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(ROOT, "tests", "ep_multi_gpu.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ep_multi_gpu: ok" in r.stdout
