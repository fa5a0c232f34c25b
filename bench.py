"""Benchmark of the MoE feed-forward layer (ornith-flight's hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload decode1|decode32|prefill4096|stack40] [--impl ours|reference]

A step = one MoE layer forward (router, softmax/top-8/renormalise, dispatch,
Q4_K/Q6_K expert SwiGLU, sigmoid-gated shared expert, weighted combine) over
one batch of synthetic tokens, on the 2048-hidden, 256-expert, top-8 layer of
BASELINE.json. Default workload: decode batch 1 (config 1).

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and torch.cuda.synchronize(), timed with CUDA events on the launching stream;
max over ranks. Step i runs layer copy i % L: L seeded layer copies (each
522 MB of expert weights, > 8 GB in total) rotate so that no step finds its
experts in the 126 MB L2 ("rotate" in config). Multi-GPU: one independent
replica per GPU (weak scaling; the decode layer has no exchange step).

The default line also carries "prefill4096" (config 3) and "stack40"
(config 4: 40 layers at batch 256, routed experts split over all N ranks,
NCCL all-to-all dispatch and combine; strong scaling, tokens/s of the whole
job) blocks measured in the same run.

--impl reference times the reference's CPU implementation of the same layer:
the reference's own engine/src/gguf.c (compiled unmodified into oracle/_ref)
for the expert dequant plus the C restatement of model.c:992-1143, on all
host cores (one process per core), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

WORKLOADS = {
    "decode1": dict(tokens=1, config="BASELINE config 1: decode batch 1", layers=16, bound="hbm",
                    dtype="f32 accumulate (int16-quantised activations, dp4a)", launches=1,
                    metric="MoE-layer tokens/s (decode batch 1)"),
    "decode32": dict(tokens=32, config="BASELINE config 2: decode batch 32", layers=16, bound="hbm",
                     dtype="f32 accumulate (int16-quantised activations, dp4a)", launches=4,
                     metric="MoE-layer tokens/s (decode batch 32)"),
    "prefill4096": dict(tokens=4096, zipf=True, layers=2, bound="tensor", dtype="bf16 (fp32 accumulate)",
                        config="BASELINE config 3: 4096-token prefill, Zipf(1.1)-skewed routing",
                        launches=7, metric="MoE-layer tokens/s (4096-token prefill)"),
    "stack40": dict(tokens=256, layers=40, bound="hbm", ep=True,
                    dtype="bf16 tensor-core / f32 dp4a experts (fp32 accumulate); rows sent bf16, results f32",
                    config="BASELINE config 4: 40-layer MoE stack, batch 256, experts sharded over the GPUs, "
                           "device-side dispatch/combine over NVLink",
                    metric="MoE-stack tokens/s (40 layers, batch 256, expert parallel)"),
}
D, H, E, K = 2048, 512, 256, 8
EXPERT_BYTES = 2 * (H * D // 256) * 144 + (H * D // 256) * 210  # 2,039,808


def algorithmic_bytes(tokens: int, n_experts_touched: int) -> int:
    # weights of the touched routed experts + shared expert + router + gate
    # vector + x in and out (decode config 1: 20,480,000 B)
    return (n_experts_touched * EXPERT_BYTES + EXPERT_BYTES + E * D * 4 + D * 4
            + 2 * tokens * D * 4)


def load_ofb():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "ornith_flight_b200.ofb", os.path.join(ROOT, "ornith-flight_b200", "ofb.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks(key):
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key]), "measured"
    except Exception:
        return fallback[key], "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU arms ---

CPU_MODES = {
    # the same layer semantics as the GPU arm: contiguous expert blocks,
    # renormalised top-8, sigmoid-gated shared expert
    "C": dict(layout=0, renorm=1, shared_gate=1,
              desc="Mode C: contiguous expert blocks, whole-block dequant, renormalised top-8, "
                   "sigmoid-gated shared expert (the GPU arm's semantics)"),
    # the reference as shipped: expert slices decoded element by element from
    # the interleaved tensors (engine/src/gguf.c:652-711), no renormalisation,
    # ungated shared expert (engine/src/model.c:992-1143)
    "R": dict(layout=1, renorm=0, shared_gate=0,
              desc="Mode R: the reference as shipped - interleaved expert slices decoded element by "
                   "element (gguf.c:652-711), top-8 without renormalisation, ungated shared expert"),
}


def _cpu_worker(args):
    """One process of the CPU arms. Builds its layer with the oracle's host
    copy of the generator (no product library is loaded in these processes)
    and runs the oracle layer, with the reference's own compiled gguf.c doing
    the dequant when oracle/_ref is built."""
    seed, seconds, tokens_per_call, use_ref, mode = args
    import binding
    if use_ref:
        binding.use_reference_dequant(True)
    m = CPU_MODES[mode]
    w = binding.make_layer_host(D, H, E, layout=m["layout"], seed=seed)
    cfg = dict(d_model=D, hidden=H, n_experts=E, top_k=K, layout=m["layout"], routing=0,
               renorm=m["renorm"], shared_gate=m["shared_gate"])
    done, t0 = 0, time.perf_counter()
    i = 0
    while True:
        x = binding.make_tokens_host(D, tokens_per_call, seed=seed * 1000 + i)
        binding.moe_forward(cfg, w, x)
        done += tokens_per_call
        i += 1
        if time.perf_counter() - t0 >= seconds:
            break
    return done, time.perf_counter() - t0


def cpu_throughput(procs: int, seconds: float, tokens_per_call: int, mode: str = "C"):
    """Tokens/s of the reference CPU layer on `procs` processes (one per core).
    The reference is single-threaded in compute; P independent processes is its
    throughput on P cores."""
    import binding
    use_ref = binding.load_ref() is not None
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        res = pool.map(_cpu_worker, [(s + 1, seconds, tokens_per_call, use_ref, mode) for s in range(procs)])
    tokens = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    kind = "reference" if use_ref else "port"
    sample = (f"{tokens} tokens ({tokens_per_call}/call) over {wall:.1f} s on {procs} process(es); "
              + CPU_MODES[mode]["desc"] + "; "
              + ("reference engine/src/gguf.c compiled unmodified (oracle/_ref) for the expert "
                 "dequant + C restatement of model.c:992-1143 (router, softmax, top-8, SwiGLU, "
                 "combine)" if use_ref else "C restatement of gguf.c dequant and model.c MoE block"))
    return tokens / wall, kind, sample


# --------------------------------------------------------------- GPU arm ----

def measure(args, ofb, dev, rank, world, local_rank, workload, steps, warmup, n_layers, sample_clocks):
    """Times `steps` layer forwards of one workload (device time, max over
    ranks), then the per-phase event times, routing paths and the end-to-end
    rate with host buffers."""
    import torch
    import torch.distributed as dist
    wl = WORKLOADS[workload]
    T = wl["tokens"]
    shape = ofb.LayerShape()
    zipf = wl.get("zipf", False)
    layers = [ofb.MoeLayer(shape, ofb.make_layer(shape, seed=1000 * rank + l, device=dev,
                                                 router_bias=ofb.zipf_bias(E, l) if zipf else None), T)
              for l in range(n_layers)]
    xs = [ofb.make_tokens(shape, T, seed=77 + i + 1000 * rank, bias_coordinate=zipf).to(dev)
          for i in range(n_layers)]
    out = torch.empty(T, D, device=dev)
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()

    def step(i):
        layers[i % n_layers].forward(xs[i % n_layers], out=out)

    for i in range(warmup):
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local_rank) if sample_clocks else None
    if clk:
        clk.__enter__()
    start.record(stream)
    for i in range(steps):
        step(i)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    if clk:
        # keep sampling for >= 1 s of identical work so that clocks are
        # observed even when K steps are shorter than one sample period
        t_extra, j = time.perf_counter(), 0
        while time.perf_counter() - t_extra < max(0.0, 1.2 - ms / 1e3):
            for _ in range(max(1, 200 // T)):
                step(j)
                j += 1
            torch.cuda.synchronize()
        clk.__exit__(None, None, None)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # per-phase device times over the same step sequence (events on the stream)
    phase = [0.0] * 4
    n_prof = min(steps, 200)
    for i in range(n_prof):
        p = layers[i % n_layers].forward_profiled(xs[i % n_layers], out)
        phase = [a + b for a, b in zip(phase, p)]
    phase = [p / n_prof for p in phase]
    route_stats = [0, 0, 0]
    for l in layers:
        route_stats = [a + b for a, b in zip(route_stats, l.ws.route_stats())]
    touched, kept = [], []
    for l in range(min(n_layers, 8)):
        idx, w = layers[l].route(xs[l])
        touched.append(len(set(idx.flatten().tolist())))
        kept.append(int((w >= 1e-6).sum().item()))

    # end to end through the public API with host buffers: every step the
    # token rows come from pinned host memory and the layer output goes back
    # to pinned host memory, moved by ofb_copy (kernel copies over the bus;
    # for decode-sized rows they beat copy-engine transfers, which are used
    # for larger batches)
    hx = [xs[i].cpu().pin_memory() for i in range(n_layers)]
    hout = torch.empty(T, D).pin_memory()
    dx = torch.empty(T, D, device=dev)
    small = T * D * 4 <= (1 << 20)

    def e2e_step(i):
        if small:
            ofb.copy(dx, hx[i % n_layers])
        else:
            dx.copy_(hx[i % n_layers], non_blocking=True)
        layers[i % n_layers].forward(dx, out=out)
        if small:
            ofb.copy(hout, out)
        else:
            hout.copy_(out, non_blocking=True)

    for i in range(warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    del layers
    torch.cuda.empty_cache()
    return dict(T=T, ms=ms, phase=phase, route_stats=route_stats, n_touched=statistics.mean(touched),
                kept=statistics.mean(kept), e2e_ms=float(te.item()), clocks=clk.summary() if clk else None)


def load_ep():
    import importlib.util
    load_ofb() if "ornith_flight_b200.ofb" not in sys.modules else None
    spec = importlib.util.spec_from_file_location(
        "ornith_flight_b200.ep", os.path.join(ROOT, "ornith-flight_b200", "ep.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def layer_launches(rows: int, tokens: int, world: int) -> int:
    """Kernels of this library one layer of the stack launches (rmsnorm
    included; the dispatch logic of moe.cu: <= 32 rows take the dp4a decode
    kernels, more the tensor-core prefill kernels)."""
    if world == 1:
        # whole layer: routing (2 certified kernels at <= 64 tokens, else 4),
        # plan + 4 tensor-core kernels, or the 2 decode kernels
        route = 2 if tokens <= 64 else 4
        return 1 + route + (2 if tokens <= 32 else 1 + 4)
    route = 2 if tokens <= 64 else 4
    shared = 1 + (3 if tokens <= 32 else 4) + 1  # gate, plan + expert kernels
    experts = 1 + 1 + 4  # unpack, plan, gather/tiles/up/down (padded rows > 32)
    return 1 + route + 1 + 1 + shared + 1 + experts + 1 + 1  # rmsnorm .. plan, dispatch, receive, return, combine


def measure_stack(args, ofb, dev, rank, world, local_rank, steps, warmup):
    """Config 4: a 40-layer stack at batch 256 with the routed experts split
    over the `world` ranks (EPStack). Device time of K stack steps, max over
    ranks; then the same with host buffers (end to end)."""
    import torch
    import torch.distributed as dist
    ep = load_ep()
    own_group = not dist.is_initialized()
    if own_group:  # one rank: a single-member NCCL group for the exchange calls
        import socket
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
        sk.close()
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                device_id=dev)
    try:
        return _measure_stack(ofb, ep, dev, rank, world, steps, warmup)
    finally:
        if own_group:
            dist.destroy_process_group()


def _measure_stack(ofb, ep, dev, rank, world, steps, warmup):
    """One rank: the whole layers (no exchange). Several ranks: EPGroup /
    EPLayerP2P, the device-side exchange over NVLink (no host sync)."""
    import ctypes
    import torch
    import torch.distributed as dist
    wl = WORKLOADS["stack40"]
    shape = ofb.LayerShape()
    T, L = wl["tokens"], wl["layers"]
    if E % world or T % world:
        raise SystemExit(f"stack40 needs the world size to divide {E} experts and {T} tokens")
    epr, tpr = E // world, T // world
    if world == 1:
        layers = [ep.LocalLayer(shape, ofb.make_layer(shape, 5000 + l, device=dev), tpr) for l in range(L)]
        group = None
    else:
        group = ep.EPGroup(shape, tpr, dev)
        layers = [ep.EPLayerP2P(shape, ofb.make_layer_slice(shape, 5000 + l, rank * epr, (rank + 1) * epr,
                                                             device=dev), group) for l in range(L)]
    stack = ep.EPStack(layers, None, tpr, dev)
    x = ofb.make_tokens(shape, T, seed=99)[rank * tpr:(rank + 1) * tpr].contiguous().to(dev)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        stack.forward(x)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        stack.forward(x)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # end to end: pinned host tokens in, final stream back, every step
    hx = x.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    dx = torch.empty_like(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(steps):
        dx.copy_(hx, non_blocking=True)
        hout.copy_(stack.forward(dx), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    errors = group.device_errors() if group else 0
    # the experts each layer routed to, for the HBM bytes: one untimed pass
    # that also routes every layer's normalised input (full router)
    ws = ofb.Workspace(shape, tpr)
    cfg = shape.config()
    idx = torch.empty(tpr, K, dtype=torch.int32, device=dev)
    wts = torch.empty(tpr, K, dtype=torch.float32, device=dev)
    xn = torch.empty_like(x)
    cur, per_layer = x, []
    for lay in layers:
        ofb._check(ofb.lib.ofb_rmsnorm(ofb._ptr(cur), tpr, D, ctypes.c_float(1e-6), ofb._ptr(xn), ofb._stream()))
        w = lay.weights if hasattr(lay, "weights") else lay.layer.weights
        ofb._check(ofb.lib.ofb_route_certified(ctypes.byref(cfg), ofb._ptr(w.router), ofb._ptr(xn), tpr,
                                               ofb._ptr(idx), ofb._ptr(wts), ws.handle, ofb._stream()))
        per_layer.append(idx.clone().reshape(-1).to(torch.int64))
        nxt = torch.empty_like(cur)
        lay.forward(xn, cur, nxt)
        cur = nxt
    all_idx = torch.stack(per_layer)  # [L][tpr*K]
    if world > 1:
        g = [torch.empty_like(all_idx) for _ in range(world)]
        dist.all_gather(g, all_idx)
        all_idx = torch.cat(g, dim=1)
    n_local = [len(set(row[(row // epr) == rank].tolist())) for row in all_idx]
    rows = [int(((row // epr) == rank).sum().item()) for row in all_idx]
    launches = sum(layer_launches(r, tpr, world) for r in rows)
    del layers, stack
    if group:
        group.close()
    torch.cuda.empty_cache()
    return dict(T=T, ms=ms, e2e_ms=float(te.item()), n_local=n_local, rows=rows, launches=launches,
                device_errors=errors)


def describe_stack(world, m, steps, warmup):
    wl = WORKLOADS["stack40"]
    T, L = m["T"], wl["layers"]
    step_ms = m["ms"] / steps
    peak, peak_kind = peaks("hbm_gbs")
    # per GPU and step: the touched local experts' weights, the replicated
    # router, shared expert and gate vector, of every layer
    gpu_bytes = sum(n * EXPERT_BYTES + EXPERT_BYTES + E * D * 4 + D * 4 for n in m["n_local"])
    achieved = gpu_bytes / (step_ms * 1e-3) / 1e9
    # rows out (bf16 on the tensor-core receive path) and results back (f32), per GPU
    nvlink = L * (T // world) * K * D * (2 + 4) * (world - 1) / world
    return {
        "metric": wl["metric"], "value": T * steps / (m["ms"] / 1e3), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "strong", "dtype": wl["dtype"],
        "data": "synthetic (seeded Q4_K/Q6_K blocks, N(0,1) tokens, N(0,0.02) router)",
        "config": {"workload": "stack40", "desc": wl["config"], "tokens_per_step": T, "layers": L,
                   "d_model": D, "hidden": H, "n_experts": E, "top_k": K, "experts_per_gpu": E // world,
                   "tokens_per_gpu": T // world, "between_layers": "unit-weight RMSNorm, residual add",
                   "exchange": "none (one rank holds every expert)" if world == 1 else
                               "device-side peer stores over NVLink with epoch-tagged flags (ofb_ep_layer_forward), "
                               "no host sync",
                   "l2": f"{L} distinct layers per step ({L * 522 // world} MB of experts per GPU) > 126 MB L2",
                   "parallelism": f"ep{world}"},
        "roofline": {"bound": "hbm", "kernel": "whole stack step (per GPU)", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                     "algorithmic_bytes_per_gpu_step": gpu_bytes},
        "nvlink_bytes_per_gpu_step": nvlink,
        "rows_received_per_layer": statistics.mean(m["rows"]),
        "e2e": {"value": T * steps / (m["e2e_ms"] / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": (T // world) * D * 4, "d2h_bytes_per_step": (T // world) * D * 4},
        "gpu_launches": m["launches"] * steps,
        "device_errors": m.get("device_errors", 0),
    }


def measure_sweep(ofb, dev, iters=20):
    """Config 5: whole-block decode of 1, 8 and 256 experts' Q4_K (gate-shaped
    512x2048) and Q6_K (down-shaped 2048x512) slices to f32 and bf16
    (ofb_dequantize over the experts' contiguous blocks, the bytes of
    gguf_dequantize_tensor_from_buf, engine/src/gguf.c:605-638). Two 256-expert
    tensors per type rotate so every call reads HBM, not L2. GB/s = (blocks
    read + values written) / device time."""
    import torch
    peak, peak_kind = peaks("hbm_gbs")
    nb = H * D // 256
    out = torch.empty(256 * nb * 256, dtype=torch.float32, device=dev)
    res = []
    for q, name, bb in ((ofb.TYPE_Q4_K, "Q4_K", 144), (ofb.TYPE_Q6_K, "Q6_K", 210)):
        srcs = [ofb.synth_blocks(q, E * nb, 900 + i, 1, device=dev) for i in range(2)]
        for n_exp in (1, 8, 256):
            for odt, osz in ((torch.float32, 4), (torch.bfloat16, 2)):
                o = out.view(torch.uint8)[: n_exp * nb * 256 * osz].view(odt)
                n_el = n_exp * nb * 256
                slices = [(s_, e0) for s_ in srcs for e0 in range(0, E, n_exp)]
                for k in range(3):
                    s_, e0 = slices[k % len(slices)]
                    ofb.dequantize(s_[e0 * nb * bb:(e0 + n_exp) * nb * bb], q, n_el, out=o)
                n_it = max(iters, min(len(slices), 512))
                torch.cuda.synchronize()
                e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e_a.record()
                for k in range(n_it):
                    s_, e0 = slices[k % len(slices)]
                    ofb.dequantize(s_[e0 * nb * bb:(e0 + n_exp) * nb * bb], q, n_el, out=o)
                e_b.record()
                torch.cuda.synchronize()
                ms = e_a.elapsed_time(e_b) / n_it
                byts = n_exp * nb * bb + n_el * osz
                gbs = byts / (ms * 1e-3) / 1e9
                res.append({"type": name, "experts": n_exp, "out": "f32" if osz == 4 else "bf16",
                            "bytes": byts, "us": ms * 1e3, "GB/s": gbs, "frac": gbs / peak})
        del srcs
    torch.cuda.empty_cache()
    return {"metric": "expert-slice dequant HBM GB/s (config 5)", "unit": "GB/s", "peak": peak,
            "peak_source": peak_kind + " hbm_gbs", "rotate": "2 tensors x 256 experts per type (>= 300 MB) > L2",
            "kernel": "q4k_dequant_kernel / q6k_dequant_kernel (bit-exact, tests/test_gpu_dequant.py)",
            "results": res}


def measure_lm_head(ofb, dev, iters=20):
    """The LM head (model.c:1219-1231): logits = x . W for an F32
    [2048][248,320] weight (2.03 GB, > L2), one token, ofb_matvec, then
    ofb_sample. GB/s = weight + x + logits bytes / device time."""
    import torch
    peak, peak_kind = peaks("hbm_gbs")
    V = 248320
    w = torch.randn(D * V, device=dev) * 0.02
    x = torch.randn(1, D, device=dev)
    out = torch.empty(1, V, device=dev)
    scratch = torch.empty(ofb.sample_scratch(V), device=dev)
    tok = torch.empty(1, dtype=torch.int32, device=dev)
    for _ in range(3):
        ofb._check(ofb.lib.ofb_matvec(ofb._ptr(x), 1, D, V, ofb._ptr(w), 0, ofb._ptr(out), ofb._stream()))
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        ofb._check(ofb.lib.ofb_matvec(ofb._ptr(x), 1, D, V, ofb._ptr(w), 0, ofb._ptr(out), ofb._stream()))
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    a.record()
    for _ in range(iters):
        ofb._check(ofb.lib.ofb_sample(ofb._ptr(out), V, 0.8, 0.5, ofb._ptr(scratch), ofb._ptr(tok), ofb._stream()))
    b.record()
    torch.cuda.synchronize()
    ms_s = a.elapsed_time(b) / iters
    byts = D * V * 4 + D * 4 + V * 4
    gbs = byts / (ms * 1e-3) / 1e9
    del w
    torch.cuda.empty_cache()
    return {"metric": "LM head GEMV (F32 2048 x 248,320, one token) + sampling", "lm_head_us": ms * 1e3,
            "GB/s": gbs, "frac": gbs / peak, "peak": peak, "peak_source": peak_kind + " hbm_gbs",
            "sample_us": ms_s * 1e3, "kernel": "matvec_kernel<F32> (bit-exact sequential sums), sample_kernel"}


def run_ours(args, rank, world, local_rank):
    import torch
    ofb = load_ofb()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    wl = WORKLOADS[args.workload]
    n_layers = args.layers if args.layers else wl["layers"]
    if wl.get("ep"):
        with ClockSampler(local_rank) as clk:
            m = measure_stack(args, ofb, dev, rank, world, local_rank, args.steps, args.warmup)
        if rank == 0:
            line = describe_stack(world, m, args.steps, args.warmup)
            line["clocks"] = clk.summary()
            print(json.dumps(line), flush=True)
        return
    m = measure(args, ofb, dev, rank, world, local_rank, args.workload, args.steps, args.warmup,
                n_layers, True)
    extra = None
    if args.workload != "prefill4096" and not args.no_prefill:
        extra = measure(args, ofb, dev, rank, world, local_rank, "prefill4096", args.prefill_steps,
                        3, WORKLOADS["prefill4096"]["layers"], False)
    d32 = None
    if args.workload == "decode1" and not args.no_decode32:
        d32 = measure(args, ofb, dev, rank, world, local_rank, "decode32", args.decode32_steps, 5,
                      WORKLOADS["decode32"]["layers"], False)
    sweep = lm = None
    if not args.no_sweep:
        sweep = measure_sweep(ofb, dev)
        lm = measure_lm_head(ofb, dev)
    stack = None
    if not args.no_stack:
        stack = measure_stack(args, ofb, dev, rank, world, local_rank, args.stack_steps, 3)
    if rank != 0:
        return
    line = describe(args, world, args.workload, m, args.steps, args.warmup, n_layers)
    if extra is not None:
        sub = describe(args, world, "prefill4096", extra, args.prefill_steps, 3,
                       WORKLOADS["prefill4096"]["layers"])
        line["prefill4096"] = {k: sub[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                                   "warmup", "config", "roofline", "layer_roofline",
                                                   "phase_ms", "e2e", "gpu_launches")}
    if d32 is not None:
        sub = describe(args, world, "decode32", d32, args.decode32_steps, 5, WORKLOADS["decode32"]["layers"])
        line["decode32"] = {k: sub[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup",
                                                "config", "roofline", "layer_roofline", "phase_ms", "e2e",
                                                "route_paths", "gpu_launches")}
    if sweep is not None:
        line["dequant_sweep"] = sweep
    if lm is not None:
        line["lm_head"] = lm
    if stack is not None:
        line["stack40"] = describe_stack(world, stack, args.stack_steps, 3)
    if not args.no_cpu_baseline:
        v, kind, sample = cpu_throughput(1, args.cpu_seconds, min(m["T"], 4))
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": 1, "kind": kind,
                                "sample": sample}
    print(json.dumps(line), flush=True)


def workload_config(workload, world, n_layers=None):
    """The config dict of a workload's line; both arms print the same one."""
    wl = WORKLOADS[workload]
    n_layers = n_layers or wl["layers"]
    return {"workload": workload, "desc": wl["config"], "tokens_per_step": wl["tokens"],
            "d_model": D, "hidden": H, "n_experts": E, "top_k": K,
            "routing": "softmax/top-8/renormalise; indices bit-exact", "shared_gate": True,
            "l2": f"rotate {n_layers} layer copies ({n_layers * 522} MB) > 126 MB L2",
            "parallelism": f"replicas x{world}"}


def describe(args, world, workload, m, steps, warmup, n_layers):
    wl = WORKLOADS[workload]
    T = m["T"]
    step_ms = m["ms"] / steps
    phase = m["phase"]
    line = {
        "metric": wl["metric"],
        "value": world * T * steps / (m["ms"] / 1e3),
        "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl["dtype"],
        "data": "synthetic (seeded Q4_K/Q6_K blocks, N(0,1) tokens, N(0,0.02) router)",
        "config": workload_config(workload, world, n_layers),
        "phase_ms": {"routing": phase[0], "plan": phase[1], "up": phase[2], "down_combine": phase[3]},
        "e2e": {"value": world * T * steps / (m["e2e_ms"] / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * D * 4, "d2h_bytes_per_step": T * D * 4},
        "route_paths": {"certified": m["route_stats"][0], "candidates_recomputed": m["route_stats"][1],
                        "all_recomputed": m["route_stats"][2]},
        "gpu_launches": (1 if T == 1 else wl["launches"]) * steps,
    }
    traffic, traffic_src = None, None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        try:
            rec = json.load(open(tp)).get(workload)
            if rec:
                traffic, traffic_src = rec["bytes"], "stored ncu capture, not measured in this run: " + rec["source"]
        except Exception:
            traffic = None
    if wl["bound"] == "hbm":
        # sub-millisecond steps: burst and sustained copy peaks are the same figure
        peak, peak_kind = peaks("hbm_gbs")
        touched = round(m["n_touched"])
        layer_bytes = algorithmic_bytes(T, touched)
        if T == 1:
            # decode batch 1 runs as one launch (decode_fused_kernel): the
            # dominant kernel is the whole layer
            # dominant kernel is the whole layer; its average launch duration is
            # the timed region's device time / K (one launch per step)
            kname, kbytes, kms = "decode_fused_kernel (whole layer, one launch)", layer_bytes, step_ms
        else:
            # the chained decode kernels: report the one with the largest share
            cands = [("route_rows_kernel + route_select_fast (router rows)", E * D * 4 + T * D * 4, phase[0]),
                     ("expert_up_q (gate/up Q4_K dequant-GEMV)", (touched + 1) * 2 * (H * D // 256) * 144, phase[2]),
                     ("expert_down_q (down Q6_K dequant-GEMV + combine)", (touched + 1) * (H * D // 256) * 210,
                      phase[3])]
            kname, kbytes, kms = max(cands, key=lambda c: c[2])
        achieved = kbytes / (kms * 1e-3) / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                            "peak_source": peak_kind + " hbm_gbs", "algorithmic_bytes_per_launch": kbytes,
                            "launch_ms": kms}
        la = layer_bytes / (step_ms * 1e-3) / 1e9
        line["layer_roofline"] = {"achieved": la, "frac": la / peak, "unit": "GB/s",
                                  "algorithmic_bytes_per_step": layer_bytes, "experts_touched": m["n_touched"]}
    else:
        # a sub-millisecond kernel timed alone: the burst GEMM peak
        peak, peak_kind = peaks("bf16_tflops")
        asg = m["kept"] + T  # routed assignments + shared expert rows
        up_flops = 4.0 * asg * H * D  # gate and up GEMMs
        achieved = up_flops / (phase[2] * 1e-3) / 1e12
        layer_flops = 6.0 * asg * H * D
        line["roofline"] = {"bound": "tensor", "kernel": "prefill_up_kernel (tcgen05 gate+up grouped GEMM)",
                            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                            "traffic": traffic, "traffic_source": traffic_src, "peak_source": peak_kind + " bf16_tflops (burst)",
                            "algorithmic_flops_per_launch": up_flops, "launch_ms": phase[2]}
        la = layer_flops / (step_ms * 1e-3) / 1e12
        line["layer_roofline"] = {"achieved": la, "frac": la / peak, "unit": "TFLOP/s",
                                  "algorithmic_flops_per_step": layer_flops}
    if m["clocks"] is not None:
        line["clocks"] = m["clocks"]
    return line


def run_reference(args, rank, world):
    """The reference arm: rank 0 times the reference's CPU layer on all host
    cores; other ranks exit without work. Headline = Mode C (the GPU arm's
    semantics); Mode R (the reference as shipped) is timed beside it."""
    if rank != 0:
        return
    procs = os.cpu_count() or 1
    wl = WORKLOADS[args.workload]
    T = wl["tokens"]
    # One token-layer takes ~0.1 s of CPU (Mode R ~0.3 s), so K steps of the
    # GPU arm's size would run for hours: each mode runs one bounded sample
    # (every core busy) and reports its throughput. The reference processes
    # one token at a time (inference.c:304-307), so its tokens/s does not
    # depend on the batch: calls of <= 4 tokens.
    v, kind, sample = cpu_throughput(procs, min(60.0, 3 * args.cpu_seconds), min(T, 4), "C")
    vr, kind_r, sample_r = cpu_throughput(procs, min(40.0, 2 * args.cpu_seconds), 1, "R")
    line = {
        "impl": "reference",
        "metric": wl["metric"], "value": v, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * T / v, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Q4_K/Q6_K blocks, N(0,1) tokens, "
                                                     "N(0,0.02) router)",
        "config": workload_config(args.workload, world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": procs, "kind": kind, "sample": sample},
        "mode_r": {"value": vr, "unit": "tokens/s", "cores": procs, "kind": kind_r, "sample": sample_r},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode1")
    ap.add_argument("--layers", type=int, default=0, help="rotating layer copies (0: workload default)")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill block of the decode line")
    ap.add_argument("--decode32-steps", type=int, default=300)
    ap.add_argument("--no-decode32", action="store_true", help="skip the decode-32 block of the decode line")
    ap.add_argument("--no-sweep", action="store_true", help="skip the dequant sweep block")
    ap.add_argument("--stack-steps", type=int, default=5)
    ap.add_argument("--no-stack", action="store_true", help="skip the expert-parallel stack block")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
