"""ofb_moe_forward_noalloc: the layer forward for callers that cannot
allocate device memory (an engine whose memory is reserved up front by its
own budget or pool, or a per-token loop that must not synchronise on
cudaMalloc/cudaFree). Its scratch is a fixed array inside the library.

Called through the C ABI and compared with ofb_moe_forward (which uses an
allocated workspace) on two calls in a row: routing indices equal, outputs
within the layer tolerance (1e-3 relative to each token's largest output).
Kept in its own file, collected last, and written to pass both on its own in
a fresh process and after the other GPU tests."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel(a, b):
    a, b = a.cpu().numpy(), b.cpu().numpy()
    return (np.abs(a - b).max(axis=1) / np.maximum(np.abs(b).max(axis=1), 1e-30)).max()


@pytest.mark.parametrize("T", [1, 4])
def test_noalloc_matches_workspace_path(ofb, cuda, T):
    shape = ofb.LayerShape()
    lw = ofb.make_layer(shape, seed=41, device=cuda)
    layer = ofb.MoeLayer(shape, lw, max_tokens=T)
    for call in range(2):
        x = ofb.make_tokens(shape, T, seed=100 + call).to(cuda)
        r = ofb.make_tokens(shape, T, seed=200 + call).to(cuda)
        i1 = torch.empty(T, shape.top_k, dtype=torch.int32, device=cuda)
        i2 = torch.empty_like(i1)
        want = layer.forward(x, r, idx=i1)
        got = layer.forward_noalloc(x, r, idx=i2)
        torch.cuda.synchronize()
        assert torch.equal(i1, i2), f"call {call}: routing differs"
        assert rel(got, want) <= TOL, f"call {call}: relative error {rel(got, want)}"


def test_noalloc_rejects_oversized_calls(ofb, cuda):
    shape = ofb.LayerShape()
    assert ofb.lib.ofb_noalloc_capacity() == 8 << 20
    lw = ofb.make_layer(shape, seed=42, device=cuda, shared=False)
    layer = ofb.MoeLayer(shape, lw, max_tokens=1)
    x = torch.zeros(512, shape.d_model, device=cuda)  # needs far more than 8 MiB
    with pytest.raises(ofb.OfbError) as ei:
        layer.forward_noalloc(x)
    assert ei.value.status == ofb.ETOOLARGE


def test_noalloc_tensor_core_batch_against_oracle(ofb, oracle, cuda):
    # 40 tokens take the tensor-core (bf16) branch and still fit the fixed
    # scratch: checked against the CPU oracle at that path's tolerance (2e-2)
    # on two calls in a row, routing indices bit-exact
    shape = ofb.LayerShape()
    T = 40
    lw = ofb.make_layer(shape, seed=43, device=cuda)
    layer = ofb.MoeLayer(shape, lw, max_tokens=1)
    cfg = dict(d_model=2048, hidden=512, n_experts=256, top_k=8, layout=0, routing=0, renorm=1, shared_gate=1)
    wd = {k: (None if v is None else v.cpu().numpy()) for k, v in vars(lw).items()}
    for call in range(2):
        x = ofb.make_tokens(shape, T, seed=300 + call)
        idx = torch.empty(T, shape.top_k, dtype=torch.int32, device=cuda)
        got = layer.forward_noalloc(x.to(cuda), idx=idx).cpu().numpy()
        want, oi, _ = oracle.moe_forward(cfg, wd, x.numpy())
        assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi), f"call {call}: routing differs"
        err = (np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)).max()
        assert err <= 2e-2, f"call {call}: relative error {err}"
