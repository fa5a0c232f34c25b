"""GGUF -> HBM loader (ofb_gguf_*): the host parser against the reference's
own gguf.c parser (oracle/_ref) on the same file — tensor types, dims,
bytes, architecture-prefixed parameters — and, on a GPU, a layer uploaded from
the file run through ofb_moe_forward against the oracle on the same bytes."""
import ctypes
import os

import numpy as np
import pytest
import torch

from gguf_writer import moe_layer_gguf

NAMES = ["ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight",
         "ffn_gate_shexp.weight", "ffn_up_shexp.weight", "ffn_down_shexp.weight", "ffn_gate_inp_shexp.weight"]


def open_gguf(ofb, path):
    h = ctypes.c_void_p()
    ofb._check(ofb.lib.ofb_gguf_open(path.encode(), ctypes.byref(h)))
    return h


def tensor(ofb, h, name):
    ty, nd = ctypes.c_int(), ctypes.c_int()
    dims = (ctypes.c_uint64 * 4)()
    off, nb = ctypes.c_uint64(), ctypes.c_uint64()
    ofb._check(ofb.lib.ofb_gguf_tensor(h, name.encode(), ctypes.byref(ty), ctypes.byref(nd), dims, ctypes.byref(off),
                                       ctypes.byref(nb)))
    return ty.value, nd.value, list(dims), off.value, nb.value


@pytest.mark.parametrize("layout", [0, 1])
def test_parser_matches_reference_gguf_c(ofb, oracle, tmp_path, layout):
    ref = oracle.load_ref()
    path = str(tmp_path / "layer.gguf")
    moe_layer_gguf(path, oracle, 512, 256, 16, 4, seed=3, layer=2, layout=layout)
    raw = open(path, "rb").read()
    h = open_gguf(ofb, path)
    try:
        for n in NAMES:
            ty, nd, dims, off, nb = tensor(ofb, h, f"blk.2.{n}")
            assert nb > 0 and off + nb <= len(raw)
            if ref is None:
                continue
            rt, rd, rsz = ctypes.c_int(), (ctypes.c_uint64 * 4)(), ctypes.c_uint64()
            buf = (ctypes.c_uint8 * nb)()
            ref.ref_gguf_tensor.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int),
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                            ctypes.POINTER(ctypes.c_uint64)]
            assert ref.ref_gguf_tensor(path.encode(), f"blk.2.{n}".encode(), ctypes.byref(rt), rd, buf, nb,
                                       ctypes.byref(rsz)) == 1
            assert (rt.value, list(rd), rsz.value) == (ty, dims, nb), n
            assert bytes(buf) == raw[off:off + nb], n
        for p, want in (("embedding_length", 512), ("expert_count", 16), ("expert_used_count", 4)):
            v = ctypes.c_uint32()
            ofb._check(ofb.lib.ofb_gguf_param_u32(h, p.encode(), ctypes.byref(v)))
            assert v.value == want
            if ref is not None:
                rv = ctypes.c_uint32()
                assert ref.ref_gguf_u32(path.encode(), p.encode(), ctypes.byref(rv)) == 1 and rv.value == want
    finally:
        ofb.lib.ofb_gguf_close(h)


def test_parser_rejects_bad_files(ofb, tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\x07\x00\x00\x00" + b"\0" * 32)  # version 7
    h = ctypes.c_void_p()
    assert ofb.lib.ofb_gguf_open(str(bad).encode(), ctypes.byref(h)) == ofb.EINVAL
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    assert ofb.lib.ofb_gguf_open(str(bad).encode(), ctypes.byref(h)) == ofb.EINVAL
    assert ofb.lib.ofb_gguf_open(str(tmp_path / "missing.gguf").encode(), ctypes.byref(h)) == ofb.EINVAL


@pytest.mark.gpu
@pytest.mark.parametrize("layout", [0, 1])
def test_uploaded_layer_matches_oracle(ofb, oracle, cuda, tmp_path, layout):
    path = str(tmp_path / "layer.gguf")
    w = moe_layer_gguf(path, oracle, 512, 256, 16, 4, seed=5, layer=0, layout=layout)
    h = open_gguf(ofb, path)
    lay = ofb.GgufMoeLayer()
    try:
        ofb._check(ofb.lib.ofb_gguf_upload_moe_layer(h, 0, layout, ctypes.byref(lay), ofb._stream()))
        cfg = lay.cfg
        assert (cfg.d_model, cfg.hidden, cfg.n_experts, cfg.top_k, cfg.shared_gate) == (512, 256, 16, 4, 1)
        T = 3
        x = oracle.make_tokens_host(512, T, seed=9)
        xd = torch.from_numpy(x).cuda()
        out = torch.empty_like(xd)
        ws = ctypes.c_void_p()
        ofb._check(ofb.lib.ofb_workspace_create(ctypes.byref(cfg), T, ctypes.byref(ws)))
        ofb._check(ofb.lib.ofb_moe_forward(ctypes.byref(cfg), ctypes.byref(lay.weights), ofb._ptr(xd), None,
                                           ofb._ptr(out), T, None, None, ws, ofb._stream()))
        torch.cuda.synchronize()
        ofb.lib.ofb_workspace_destroy(ws)
        want, _, _ = oracle.moe_forward(dict(d_model=512, hidden=256, n_experts=16, top_k=4, layout=layout,
                                             routing=0, renorm=1, shared_gate=1), w, x)
        got = out.cpu().numpy()
        err = (np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)).max()
        assert err <= 1e-3, err
    finally:
        ofb.lib.ofb_gguf_free_moe_layer(ctypes.byref(lay))
        ofb.lib.ofb_gguf_close(h)
