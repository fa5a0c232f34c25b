"""The oracle's MoE layer against an independent float64 numpy model of the
same math (routing indices exact away from near-ties; outputs to 1e-4)."""
import numpy as np
import pytest


def np_layer(cfg, w, x, deq):
    D, H, E, K = cfg["d_model"], cfg["hidden"], cfg["n_experts"], cfg["top_k"]
    W = w["router"].reshape(E, D).astype(np.float64)
    nb = H * D // 256
    outs, idxs = [], []
    for t in range(x.shape[0]):
        xt = x[t].astype(np.float64)
        lg = W @ xt
        p = np.exp(lg - lg.max()); p /= p.sum()
        idx = np.argsort(-p, kind="stable")[:K]
        pw = p[idx] / p[idx].sum() if cfg["renorm"] else p[idx]
        o = np.zeros(D)

        def expert(g, u, dn):
            G = deq(g, 12, H * D).reshape(H, D); U = deq(u, 12, H * D).reshape(H, D)
            Dn = deq(dn, 14, H * D).reshape(D, H)
            gg, uu = G @ xt, U @ xt
            s = np.where(gg < -50, 0, np.where(gg > 50, gg, gg / (1 + np.exp(-gg))))
            return Dn @ (s * uu)

        ysh = expert(w["gate_shexp"], w["up_shexp"], w["down_shexp"])
        gate = 1 / (1 + np.exp(-(xt @ w["shexp_gate"].astype(np.float64)))) if cfg["shared_gate"] else 1.0
        o += gate * ysh
        for a, e in enumerate(idx):
            o += pw[a] * expert(w["gate_exps"][e * nb * 144:(e + 1) * nb * 144],
                                w["up_exps"][e * nb * 144:(e + 1) * nb * 144],
                                w["down_exps"][e * nb * 210:(e + 1) * nb * 210])
        outs.append(o); idxs.append(idx)
    return np.array(outs), np.array(idxs)


@pytest.mark.parametrize("renorm,gate", [(1, 1), (0, 0)])
def test_oracle_layer_vs_float64(ofb, oracle, renorm, gate):
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=16, top_k=4, renorm=renorm, shared_gate=gate)
    lw = ofb.make_layer(shape, seed=11, device="cpu")
    x = ofb.make_tokens(shape, 6, seed=11).numpy()
    cfg = dict(d_model=512, hidden=256, n_experts=16, top_k=4, layout=0, routing=0, renorm=renorm,
               shared_gate=gate)
    w = {k: (None if v is None else v.numpy()) for k, v in vars(lw).items()}
    out, idx, wt = oracle.moe_forward(cfg, w, x)
    ref, ridx = np_layer(cfg, w, x, lambda b, q, n: oracle.dequant(b, q, n).astype(np.float64))
    assert np.array_equal(idx.astype(np.int64), ridx)
    err = np.abs(out - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() < 1e-4, err
