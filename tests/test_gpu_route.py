"""Device routing bit-exact against the reference's CPU routing (oracle):
indices and weights, both routing variants, both router layouts, decode and
prefill token counts, ties, the uniform fallback, and the device expf."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def oracle_route(oracle, cfg, router, x):
    # the oracle layer call returns routing; use a no-shared, tiny-expert layer
    import binding
    o = binding.orc()
    T, D = x.shape
    c = binding.OrcCfg(D, 256, cfg["n_experts"], cfg["top_k"], cfg["layout"], cfg["routing"], cfg["renorm"], 0)
    idx = np.empty((T, cfg["top_k"]), np.uint32)
    w = np.empty((T, cfg["top_k"]), np.float32)
    import ctypes
    o.orc_route_token.restype = None
    o.orc_route_token.argtypes = [ctypes.POINTER(binding.OrcCfg), ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_void_p]
    xr = np.ascontiguousarray(x, np.float32)
    rr = None if router is None else np.ascontiguousarray(router, np.float32)
    for t in range(T):
        o.orc_route_token(ctypes.byref(c), xr[t].ctypes.data, None if rr is None else rr.ctypes.data,
                          idx[t].ctypes.data, w[t].ctypes.data)
    return idx, w


def run(ofb, cuda, shape, router, x):
    lw = ofb.LayerWeights(None if router is None else torch.from_numpy(router).to(cuda),
                          torch.zeros(16, dtype=torch.uint8, device=cuda),
                          torch.zeros(16, dtype=torch.uint8, device=cuda),
                          torch.zeros(16, dtype=torch.uint8, device=cuda), None, None, None, None)
    layer = ofb.MoeLayer(shape, lw, max_tokens=x.shape[0])
    idx, w = layer.route(torch.from_numpy(x).to(cuda))
    return idx.cpu().numpy().view(np.uint32), w.cpu().numpy()


CASES = [(1, 0, 0, 1), (32, 0, 0, 1), (4096, 0, 0, 1), (7, 1, 0, 0), (100, 0, 1, 0), (33, 1, 1, 0)]


@pytest.mark.parametrize("T,layout,routing,renorm", CASES)
def test_routing_bit_exact(ofb, oracle, cuda, T, layout, routing, renorm):
    E, D, K = 256, 2048, 8
    shape = ofb.LayerShape(d_model=D, hidden=256, n_experts=E, top_k=K, layout=layout,
                           routing=routing, renorm=renorm)
    router = ofb.synth_normal(E * D, 0, 7, 0.02).numpy()
    x = ofb.make_tokens(shape, T, seed=T).numpy()
    gi, gw = run(ofb, cuda, shape, router, x)
    cfg = dict(n_experts=E, top_k=K, layout=layout, routing=routing, renorm=renorm)
    oi, ow = oracle_route(oracle, cfg, router, x)
    assert np.array_equal(gi, oi)
    assert np.array_equal(gw.view(np.uint32), ow.view(np.uint32))


@pytest.mark.parametrize("routing", [0, 1])
def test_routing_ties_follow_exchange_sort(ofb, oracle, cuda, routing):
    # duplicated router rows give exactly equal logits (and probabilities):
    # the exchange sort's swap order decides which duplicate comes first.
    E, D, K = 64, 256, 8
    rng = np.random.default_rng(1)
    base = rng.normal(0, 0.02, size=(8, D)).astype(np.float32)
    router = base[rng.integers(0, 8, size=E)]
    shape = ofb.LayerShape(d_model=D, hidden=256, n_experts=E, top_k=K, routing=routing)
    x = rng.normal(size=(50, D)).astype(np.float32)
    gi, gw = run(ofb, cuda, shape, router.reshape(-1), x)
    oi, ow = oracle_route(oracle, dict(n_experts=E, top_k=K, layout=0, routing=routing, renorm=1),
                          router.reshape(-1), x)
    assert np.array_equal(gi, oi)
    assert np.array_equal(gw.view(np.uint32), ow.view(np.uint32))


def test_uniform_fallback_without_router(ofb, oracle, cuda):
    shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=16, top_k=4)
    x = np.ones((3, 256), np.float32)
    gi, gw = run(ofb, cuda, shape, None, x)
    assert np.array_equal(gi, np.tile(np.arange(4, dtype=np.uint32), (3, 1)))
    assert np.all(gw == np.float32(1.0) / np.float32(4))


def test_small_expert_counts_and_k_equals_e(ofb, oracle, cuda):
    for E, K in ((1, 1), (3, 3), (40, 16)):
        shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=E, top_k=K)
        router = ofb.synth_normal(E * 256, 1, 7, 0.1).numpy()
        x = ofb.make_tokens(shape, 9, seed=E).numpy()
        gi, gw = run(ofb, cuda, shape, router, x)
        oi, ow = oracle_route(oracle, dict(n_experts=E, top_k=K, layout=0, routing=0, renorm=1), router, x)
        assert np.array_equal(gi, oi) and np.array_equal(gw.view(np.uint32), ow.view(np.uint32))


def test_device_expf_matches_host(ofb, oracle, cuda):
    # softmax on logits crafted so that l - max sweeps a strided sample of all
    # non-positive floats: the returned GET_ROUTING weights are expf(l - max)/sum
    # with sum == expf(0) == 1 when top_k == 1 ... instead compare probabilities
    # of a FORWARD softmax with every expert kept (top_k == E), renorm off.
    E = 64
    rng = np.random.default_rng(0)
    bits = np.sort(rng.integers(0x80000000, 0xC3000000, size=E * 200, dtype=np.uint64)).astype(np.uint32)
    deltas = bits.view(np.float32).reshape(200, E)
    deltas[:, 0] = 0.0
    shape = ofb.LayerShape(d_model=256, hidden=256, n_experts=E, top_k=16, routing=0, renorm=0)
    # x = e_0 one-hot => logit[e] = W[e][0]
    router = np.zeros((E, 256), np.float32)
    for r in range(200):
        router[:, 0] = deltas[r]
        x = np.zeros((1, 256), np.float32); x[0, 0] = 1.0
        gi, gw = run(ofb, cuda, shape, router.reshape(-1), x)
        oi, ow = oracle_route(oracle, dict(n_experts=E, top_k=16, layout=0, routing=0, renorm=0),
                              router.reshape(-1), x)
        assert np.array_equal(gi, oi) and np.array_equal(gw.view(np.uint32), ow.view(np.uint32))
