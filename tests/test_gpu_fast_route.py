"""The certified routing inside ofb_moe_forward (contiguous router): top-k
indices bit-exact against the reference's sequential CPU routing on every
path — certified directly, uncertain candidates recomputed with the exact
chain, and every logit recomputed (probability ties) — at decode sizes
(T <= 64: route_rows / route_select_fast) and above (bounded GEMM,
route_certify_warps, route_fallback_warps)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def run_layer(ofb, oracle, cuda, shape, router, x):
    lw = ofb.make_layer(shape, seed=3, device=cuda)
    lw.router = torch.from_numpy(np.ascontiguousarray(router, np.float32).reshape(-1)).to(cuda)
    T = x.shape[0]
    layer = ofb.MoeLayer(shape, lw, max_tokens=T)
    idx = torch.empty(T, shape.top_k, dtype=torch.int32, device=cuda)
    w = torch.empty(T, shape.top_k, dtype=torch.float32, device=cuda)
    out = layer.forward(torch.from_numpy(x).to(cuda), idx=idx, w=w)
    torch.cuda.synchronize()
    cfg = dict(d_model=shape.d_model, hidden=shape.hidden, n_experts=shape.n_experts, top_k=shape.top_k,
               layout=0, routing=shape.routing, renorm=shape.renorm, shared_gate=shape.shared_gate)
    wd = {k: (None if v is None else v.cpu().numpy()) for k, v in vars(lw).items()}
    want, oi, ow = oracle.moe_forward(cfg, wd, x)
    return idx.cpu().numpy().view(np.uint32), w.cpu().numpy(), out.cpu().numpy(), oi, ow, want, \
        layer.ws.route_stats()


@pytest.mark.parametrize("routing", [0, 1])
def test_many_tokens_certified(ofb, oracle, cuda, routing):
    shape = ofb.LayerShape(routing=routing)
    router = ofb.synth_normal(256 * 2048, 0, 7, 0.02).numpy().reshape(256, 2048)
    x = ofb.make_tokens(shape, 64, seed=123).numpy()
    gi, gw, out, oi, ow, want, stats = run_layer(ofb, oracle, cuda, shape, router, x)
    assert np.array_equal(gi, oi)
    np.testing.assert_allclose(gw, ow, rtol=1e-5)
    assert stats[0] > 0 and sum(stats) == 64


def test_near_ties_recompute_candidates(ofb, oracle, cuda):
    # expert pairs whose logits differ by ~1e-6 relative: inside the error
    # bound, so the block recomputes them with the reference's exact chain
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=32, top_k=4)
    rng = np.random.default_rng(4)
    base = rng.normal(0, 0.05, size=(16, 512)).astype(np.float32)
    router = np.concatenate([base, base * np.float32(1 + 3e-6)])
    x = rng.normal(size=(40, 512)).astype(np.float32)
    gi, gw, out, oi, ow, want, stats = run_layer(ofb, oracle, cuda, shape, router, x)
    assert np.array_equal(gi, oi)
    np.testing.assert_allclose(gw, ow, rtol=1e-5)
    assert stats[1] + stats[2] > 0


@pytest.mark.parametrize("routing", [0, 1])
def test_exact_ties_full_recompute(ofb, oracle, cuda, routing):
    # duplicated rows: equal logits; the exchange sort's swap order decides
    shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=48, top_k=8, routing=routing)
    rng = np.random.default_rng(5)
    base = rng.normal(0, 0.05, size=(6, 256)).astype(np.float32)
    router = base[rng.integers(0, 6, size=48)]
    x = rng.normal(size=(30, 256)).astype(np.float32)
    gi, gw, out, oi, ow, want, stats = run_layer(ofb, oracle, cuda, shape, router, x)
    assert np.array_equal(gi, oi)
    np.testing.assert_allclose(gw, ow, rtol=1e-5)
    if routing == 0:
        assert stats[2] > 0  # probabilities tie -> every logit recomputed


@pytest.mark.parametrize("routing", [0, 1])
def test_large_batch_exact_ties_warp_fallback(ofb, oracle, cuda, routing):
    # above 64 tokens: bounded GEMM + warp certificate; duplicated router rows
    # leave every token to route_fallback_warps, whose forward-routing
    # probabilities tie and so recompute every logit
    shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=48, top_k=8, routing=routing)
    rng = np.random.default_rng(15)
    base = rng.normal(0, 0.05, size=(6, 256)).astype(np.float32)
    router = base[rng.integers(0, 6, size=48)]
    x = rng.normal(size=(100, 256)).astype(np.float32)
    gi, gw, out, oi, ow, want, stats = run_layer(ofb, oracle, cuda, shape, router, x)
    assert np.array_equal(gi, oi)
    np.testing.assert_allclose(gw, ow, rtol=1e-5)
    assert stats[0] + stats[1] + stats[2] == 100
    if routing == 0:
        assert stats[2] > 0


def test_large_batch_near_ties_warp_fallback(ofb, oracle, cuda):
    # near-equal expert pairs above 64 tokens: candidates recomputed by the
    # warp fallback with the reference's exact chain
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=32, top_k=4)
    rng = np.random.default_rng(14)
    base = rng.normal(0, 0.05, size=(16, 512)).astype(np.float32)
    router = np.concatenate([base, base * np.float32(1 + 3e-6)])
    x = rng.normal(size=(120, 512)).astype(np.float32)
    gi, gw, out, oi, ow, want, stats = run_layer(ofb, oracle, cuda, shape, router, x)
    assert np.array_equal(gi, oi)
    np.testing.assert_allclose(gw, ow, rtol=1e-5)
    assert stats[1] + stats[2] > 0


@pytest.mark.parametrize("T,routing,bias", [(1, 0, False), (17, 1, False), (64, 0, True), (65, 0, False),
                                            (300, 1, False), (1000, 0, True)])
def test_route_certified_entry(ofb, cuda, T, routing, bias):
    """ofb_route_certified (decode-size and large-batch certified paths)
    against ofb_route (the exact reference routing): indices identical,
    weights within 1e-5 relative; the Zipf-biased router pushes near-ties."""
    import ctypes
    shape = ofb.LayerShape(routing=routing)
    r = ofb.make_router(shape, 5, ofb.zipf_bias(shape.n_experts, 5) if bias else None).to(cuda)
    x = ofb.make_tokens(shape, T, seed=T, bias_coordinate=bias).to(cuda)
    ws = ofb.Workspace(shape, T)
    cfg = shape.config()
    res = []
    for fn in (ofb.lib.ofb_route, ofb.lib.ofb_route_certified):
        idx = torch.empty(T, shape.top_k, dtype=torch.int32, device=cuda)
        w = torch.empty(T, shape.top_k, dtype=torch.float32, device=cuda)
        ofb._check(fn(ctypes.byref(cfg), ofb._ptr(r), ofb._ptr(x), T, ofb._ptr(idx), ofb._ptr(w), ws.handle,
                      ofb._stream()))
        torch.cuda.synchronize()
        res.append((idx.cpu().numpy(), w.cpu().numpy()))
    assert np.array_equal(res[0][0], res[1][0])
    np.testing.assert_allclose(res[1][1], res[0][1], rtol=1e-5)
