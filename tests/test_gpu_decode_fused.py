"""Decode batch 1 through ofb_moe_forward: the single-launch layer kernel
(decode_fused.cu) against the oracle's restatement of
engine/src/model.c:992-1143 for one token.

Tolerances: top-k indices bit-exact; weights within 1e-5 relative (certified
routing; bit-exact when every logit is recomputed); layer output per token
max|gpu - ref| <= 1e-3 * max|ref| (fp32 accumulate, 16-bit quantised
activations). Every routing path of the kernel is forced: certified, exact
recompute of near-tied candidates, and the full recompute when probabilities
tie."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-3
WEIGHT_RTOL = 1e-5
SMALL = dict(d_model=512, hidden=256, n_experts=16, top_k=4)


def cfg_of(shape):
    return dict(d_model=shape.d_model, hidden=shape.hidden, n_experts=shape.n_experts, top_k=shape.top_k,
                layout=shape.layout, routing=shape.routing, renorm=shape.renorm, shared_gate=shape.shared_gate)


def run_tokens(ofb, oracle, cuda, shape, lw, xs, resid=None, errors=False):
    """One T = 1 call per token on one layer; returns the worst relative error
    and the routing stats; asserts indices / weights per token."""
    layer = ofb.MoeLayer(shape, lw, max_tokens=1)
    wd = {k: (None if v is None else v.cpu().numpy()) for k, v in vars(lw).items()}
    worst = 0.0
    for t in range(xs.shape[0]):
        x = xs[t:t + 1]
        r = None if resid is None else resid[t:t + 1]
        idx = torch.empty(1, shape.top_k, dtype=torch.int32, device=cuda)
        w = torch.empty(1, shape.top_k, dtype=torch.float32, device=cuda)
        out = layer.forward(torch.from_numpy(x).to(cuda), None if r is None else torch.from_numpy(r).to(cuda),
                            idx=idx, w=w)
        want, oi, ow = oracle.moe_forward(cfg_of(shape), wd, x, r)
        got = out.cpu().numpy()
        assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi), f"token {t}: indices differ"
        np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=WEIGHT_RTOL, atol=0, err_msg=f"token {t}")
        err = np.abs(got - want).max() / np.abs(want).max()
        worst = max(worst, err)
        assert err <= TOL, f"token {t}: relative error {err}"
    if errors:
        torch.cuda.synchronize()
        return worst, layer.ws.route_stats(), layer.ws.device_errors()
    return worst, layer.ws.route_stats()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_config1_layer_many_tokens(ofb, oracle, cuda, seed):
    # the BASELINE config-1 layer, 6 tokens per seed, one call each (the
    # epoch-tagged exchange words are reused across calls)
    shape = ofb.LayerShape()
    lw = ofb.make_layer(shape, seed=40 + seed, device=cuda)
    xs = ofb.make_tokens(shape, 6, seed=90 + seed).numpy()
    worst, stats = run_tokens(ofb, oracle, cuda, shape, lw, xs)
    assert sum(stats) == 6


@pytest.mark.parametrize("renorm,gate,routing", [(0, 0, 0), (1, 0, 0), (0, 1, 1), (1, 1, 1)])
def test_modes_with_residual(ofb, oracle, cuda, renorm, gate, routing):
    shape = ofb.LayerShape(**SMALL, renorm=renorm, shared_gate=gate, routing=routing)
    lw = ofb.make_layer(shape, seed=5, device=cuda)
    xs = ofb.make_tokens(shape, 4, seed=6).numpy()
    rs = ofb.make_tokens(shape, 4, seed=7).numpy()
    run_tokens(ofb, oracle, cuda, shape, lw, xs, rs)


def test_no_shared_expert(ofb, oracle, cuda):
    shape = ofb.LayerShape(**SMALL)
    lw = ofb.make_layer(shape, seed=8, device=cuda, shared=False)
    run_tokens(ofb, oracle, cuda, shape, lw, ofb.make_tokens(shape, 3, seed=9).numpy())


@pytest.mark.parametrize("d_model,hidden,n_experts,top_k", [(1024, 512, 64, 6), (2048, 768, 128, 8),
                                                            (4096, 1024, 256, 16), (256, 256, 8, 2)])
def test_other_shapes(ofb, oracle, cuda, d_model, hidden, n_experts, top_k):
    shape = ofb.LayerShape(d_model=d_model, hidden=hidden, n_experts=n_experts, top_k=top_k)
    lw = ofb.make_layer(shape, seed=11, device=cuda)
    run_tokens(ofb, oracle, cuda, shape, lw, ofb.make_tokens(shape, 2, seed=12).numpy())


def test_near_ties_recompute_candidates(ofb, oracle, cuda):
    # expert pairs whose logits differ by ~1e-6 relative: inside the bound,
    # so every CTA recomputes them with the reference's exact chain
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=32, top_k=4)
    rng = np.random.default_rng(4)
    base = rng.normal(0, 0.05, size=(16, 512)).astype(np.float32)
    router = np.concatenate([base, base * np.float32(1 + 3e-6)])
    lw = ofb.make_layer(shape, seed=3, device=cuda)
    lw.router = torch.from_numpy(router.reshape(-1)).to(cuda)
    xs = rng.normal(size=(12, 512)).astype(np.float32)
    _, stats, errs = run_tokens(ofb, oracle, cuda, shape, lw, xs, errors=True)
    assert stats[1] + stats[2] > 0
    assert errs == 0  # no bounded wait expired on the recompute path


@pytest.mark.parametrize("routing", [0, 1])
def test_exact_ties_full_recompute(ofb, oracle, cuda, routing):
    # duplicated router rows: equal logits; the exchange sort's swap order
    # decides, and forward routing's tied probabilities recompute everything
    shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=48, top_k=8, routing=routing)
    rng = np.random.default_rng(5)
    base = rng.normal(0, 0.05, size=(6, 256)).astype(np.float32)
    router = base[rng.integers(0, 6, size=48)]
    lw = ofb.make_layer(shape, seed=3, device=cuda)
    lw.router = torch.from_numpy(np.ascontiguousarray(router).reshape(-1)).to(cuda)
    xs = rng.normal(size=(8, 256)).astype(np.float32)
    _, stats, errs = run_tokens(ofb, oracle, cuda, shape, lw, xs, errors=True)
    if routing == 0:
        assert stats[2] > 0
    assert errs == 0


def test_back_to_back_calls_in_one_stream(ofb, oracle, cuda):
    # many launches queued without host synchronisation (dependent launches
    # overlap the next call's static loads with the previous call's tail);
    # every output is kept and checked afterwards
    shape = ofb.LayerShape()
    layers = [ofb.make_layer(shape, seed=60 + i, device=cuda) for i in range(2)]
    mls = [ofb.MoeLayer(shape, lw, max_tokens=1) for lw in layers]
    xs = ofb.make_tokens(shape, 10, seed=61).numpy()
    outs = []
    for t in range(10):
        outs.append(mls[t % 2].forward(torch.from_numpy(xs[t:t + 1]).to(cuda)))
    torch.cuda.synchronize()
    for t in range(10):
        lw = layers[t % 2]
        wd = {k: (None if v is None else v.cpu().numpy()) for k, v in vars(lw).items()}
        want, _, _ = oracle.moe_forward(cfg_of(shape), wd, xs[t:t + 1])
        err = np.abs(outs[t].cpu().numpy() - want).max() / np.abs(want).max()
        assert err <= TOL, f"call {t}: relative error {err}"


def test_no_device_errors_recorded(ofb, cuda):
    shape = ofb.LayerShape(**SMALL)
    lw = ofb.make_layer(shape, seed=2, device=cuda)
    layer = ofb.MoeLayer(shape, lw, max_tokens=1)
    for t in range(3):
        layer.forward(ofb.make_tokens(shape, 1, seed=t).to(cuda))
    torch.cuda.synchronize()
    assert layer.ws.device_errors() == 0
