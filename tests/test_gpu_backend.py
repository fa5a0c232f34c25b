"""The gpu.h CUDA backend: the reference's own backend contract tests
(engine/test/t_gpu.c, t_gpu_metal.c, linked against libornith_cuda.so by
`make -C oracle` when the reference tree is present) and the MoE-related
gpu.h calls through ctypes against the oracle."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "ornith-flight_b200", "libornith_cuda.so")


@pytest.mark.parametrize("binary", ["t_gpu_cuda", "t_gpu_metal_cuda"])
def test_reference_backend_contract(cuda, binary):
    exe = os.path.join(ROOT, "oracle", "_ref", binary)
    if not os.path.exists(exe):
        pytest.skip(f"{binary} not built (needs the reference tree at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


class Backend:
    def __init__(self):
        L = ctypes.CDLL(LIB)
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        L.gpu_init.restype = vp
        L.gpu_destroy.argtypes = [vp]
        L.gpu_alloc.restype, L.gpu_alloc.argtypes = vp, [vp, sz, i32]
        L.gpu_free.argtypes = [vp, vp]
        L.gpu_copy_to_device.argtypes = [vp, vp, vp, sz]
        L.gpu_copy_to_host.argtypes = [vp, vp, vp, sz]
        L.gpu_router.argtypes = [vp, vp, vp, vp, i32, i32]
        L.gpu_topk_softmax.argtypes = [vp, vp, vp, vp, i32, i32]
        L.gpu_expert_mlp.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32]
        L.gpu_last_error.restype, L.gpu_last_error.argtypes = i32, [vp]
        L.gpu_memory_used.restype, L.gpu_memory_used.argtypes = sz, [vp]
        self.L = L
        self.ctx = L.gpu_init()
        assert self.ctx

    def upload(self, a: np.ndarray):
        a = np.ascontiguousarray(a)
        b = self.L.gpu_alloc(self.ctx, a.nbytes, 0)
        self.L.gpu_copy_to_device(self.ctx, b, a.ctypes.data, a.nbytes)
        return b

    def download(self, b, shape, dtype):
        out = np.empty(shape, dtype)
        self.L.gpu_copy_to_host(self.ctx, out.ctypes.data, b, out.nbytes)
        return out


def test_router_and_topk_match_oracle(cuda, oracle):
    be = Backend()
    D, E, K = 2048, 256, 8
    rng = np.random.default_rng(5)
    W = rng.normal(0, 0.02, size=(D, E)).astype(np.float32)  # [D][E] (mlp.metal:94-109)
    x = rng.normal(size=D).astype(np.float32)
    bW, bx = be.upload(W), be.upload(x)
    bl = be.L.gpu_alloc(be.ctx, E * 4, 0)
    be.L.gpu_router(be.ctx, bl, bx, bW, D, E)
    logits = be.download(bl, E, np.float32)
    want = np.zeros(E, np.float32)
    for e in range(E):  # sequential fp32, same order as the reference
        s = np.float32(0)
        for d in range(D):
            s = np.float32(s + np.float32(x[d] * W[d, e]))
        want[e] = s
    assert np.array_equal(logits.view(np.uint32), want.view(np.uint32))
    idx = np.empty(K, np.uint32)
    w = np.empty(K, np.float32)
    be.L.gpu_topk_softmax(be.ctx, idx.ctypes.data, w.ctypes.data, bl, E, K)
    order = np.argsort(-want, kind="stable")[:K]
    assert np.array_equal(idx, order.astype(np.uint32))
    ex = np.array([oracle.orc().orc_expf(float(v - want[order[0]])) for v in want[order]], np.float32)
    s = np.float32(0)
    for v in ex:
        s = np.float32(s + v)
    assert np.array_equal(w.view(np.uint32), (ex / s).astype(np.float32).view(np.uint32))
    assert be.L.gpu_last_error(be.ctx) == 0
    be.L.gpu_destroy(be.ctx)


def test_expert_mlp_q4k(cuda, ofb, oracle):
    be = Backend()
    shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=1, top_k=1, shared_gate=0, renorm=0)
    lw = ofb.make_layer(shape, seed=2, device="cpu", shared=False, router=False)
    x = ofb.make_tokens(shape, 1, seed=3).numpy()
    bg, bu, bd = (be.upload(t.numpy()) for t in (lw.gate_exps, lw.up_exps, lw.down_exps))
    bx = be.upload(x)
    bo = be.L.gpu_alloc(be.ctx, 512 * 4, 0)
    be.L.gpu_expert_mlp(be.ctx, bo, bx, bg, bu, bd, 512, 256, 4)  # QUANT_Q4_K
    got = be.download(bo, (1, 512), np.float32)
    w = {k: (None if v is None else v.numpy()) for k, v in vars(lw).items()}
    cfg = dict(d_model=512, hidden=256, n_experts=1, top_k=1, layout=0, routing=0, renorm=0, shared_gate=0)
    want, _, _ = oracle.moe_forward(cfg, w, x)
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    be.L.gpu_destroy(be.ctx)


def test_null_arguments_are_silent(cuda):
    be = Backend()
    be.L.gpu_router(be.ctx, None, None, None, 4, 4)
    be.L.gpu_expert_mlp(be.ctx, None, None, None, None, None, 4, 4, 0)
    assert be.L.gpu_alloc(be.ctx, 0, 0) is None
    assert be.L.gpu_memory_used(be.ctx) == 0
    be.L.gpu_destroy(be.ctx)
