"""Dense projections on the raw GGUF tensors (ofb_matvec), the LM head and
sampling (ofb_sample), and gpu_matmul with a block-quantised B, against the
reference's arithmetic: the weight dequantised with the reference's own
per-element rule (oracle) and multiplied with its sequential fp32 sum
(orc_matmul = gpu.c's / cpu_matmul_vec's order, no FMA). Matvec and LM-head
outputs are bit-exact; sampling matches a float64 restatement except within
the rounding distance of a cumulative-probability boundary."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def ref_matmul(oracle, A, B):
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    oracle.orc().orc_matmul(C.ctypes.data, np.ascontiguousarray(A).ctypes.data,
                            np.ascontiguousarray(B).ctypes.data, M, N, K)
    return C


@pytest.mark.parametrize("wt,in_dim,out_dim,T", [(12, 512, 768, 1), (14, 768, 512, 3), (1, 256, 1000, 5),
                                                 (0, 300, 777, 2), (12, 2048, 4096, 1)])
def test_matvec_bit_exact(ofb, oracle, cuda, wt, in_dim, out_dim, T):
    rng = np.random.default_rng(wt + T)
    n = in_dim * out_dim
    if wt in (12, 14):
        blocks = ofb.synth_blocks_host(wt, n // 256, seed=wt, stream_id=T).numpy()
    elif wt == 1:
        blocks = rng.integers(0, 0x7BFF, size=n, dtype=np.int32).astype(np.uint16).view(np.uint8)
    else:
        blocks = rng.normal(size=n).astype(np.float32).view(np.uint8)
    W = oracle.dequant(blocks, wt, n).reshape(in_dim, out_dim)
    x = rng.normal(size=(T, in_dim)).astype(np.float32)
    got = ofb.matvec(torch.from_numpy(x).to(cuda), torch.from_numpy(blocks.copy()).to(cuda), wt, out_dim).cpu().numpy()
    want = ref_matmul(oracle, x, W)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_lm_head_full_vocab_bit_exact(ofb, oracle, cuda):
    # model.c:1219-1231: output[i] = sum_d x[d] * w[d * vocab + i], vocab 248,320
    D, V = 2048, 248320
    w = ofb.synth_normal(D * V, seed=1, stream_id=21, sigma=0.02).numpy()
    x = np.random.default_rng(2).normal(size=(1, D)).astype(np.float32)
    got = ofb.matvec(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), 0, V).cpu().numpy()
    want = ref_matmul(oracle, x, w.reshape(D, V))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("temp", [1.0, 0.7, 0.0])
def test_sample_matches_reference_cumulative_rule(ofb, cuda, temp):
    V = 248320
    rng = np.random.default_rng(3)
    logits = (rng.normal(size=V) * 3).astype(np.float32)
    dl = torch.from_numpy(logits).to(cuda)
    l64 = logits.astype(np.float64) / (temp if temp > 0 and temp != 1.0 else 1.0)
    p = np.exp(l64 - l64.max())
    cum = np.cumsum(p / p.sum())
    for r in rng.uniform(0, 1, size=40):
        tok = ofb.sample(dl, temp, float(r))
        want = int(np.searchsorted(cum, r))
        if tok != want:
            # only allowed where r sits within rounding distance of a boundary
            assert abs(cum[min(tok, want)] - r) < V * 2.0 ** -24, (tok, want, r)


@pytest.mark.parametrize("V", [1, 7, 1024, 1025, 3000, 70001])
def test_sample_ragged_vocab_and_edges(ofb, cuda, V):
    # chunk edges (1024 logits per CTA), r = 0 (index 0) and r above every
    # cumulative sum (the reference's vocab - 1)
    rng = np.random.default_rng(V)
    logits = (rng.normal(size=V) * 2).astype(np.float32)
    dl = torch.from_numpy(logits).to(cuda)
    p = np.exp(logits.astype(np.float64) - logits.max())
    cum = np.cumsum(p / p.sum())
    assert ofb.sample(dl, 1.0, 0.0) == 0
    assert ofb.sample(dl, 1.0, 1.5) == V - 1
    for r in rng.uniform(0, 1, size=20):
        tok = ofb.sample(dl, 1.0, float(r))
        want = min(int(np.searchsorted(cum, r)), V - 1)
        if tok != want:
            assert abs(cum[min(tok, want)] - r) < max(V, 1024) * 2.0 ** -24, (tok, want, r)


def test_gpu_matmul_quantised_b(ofb, oracle, cuda):
    L = ctypes.CDLL(ofb.LIB_PATH)
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.gpu_init.restype = vp
    L.gpu_alloc.restype, L.gpu_alloc.argtypes = vp, [vp, sz, i32]
    L.gpu_copy_to_device.argtypes = [vp, vp, vp, sz]
    L.gpu_copy_to_host.argtypes = [vp, vp, vp, sz]
    L.gpu_matmul.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32]
    L.gpu_last_error.restype, L.gpu_last_error.argtypes = i32, [vp]
    L.gpu_destroy.argtypes = [vp]
    ctx = L.gpu_init()
    M, K, N = 3, 512, 1024
    QUANT_Q4_K, QUANT_Q6_K = 4, 5
    for q, wt in ((QUANT_Q4_K, 12), (QUANT_Q6_K, 14)):
        blocks = ofb.synth_blocks_host(wt, K * N // 256, seed=7, stream_id=q).numpy()
        A = np.random.default_rng(q).normal(size=(M, K)).astype(np.float32)
        bufs = []
        for arr in (A, blocks):
            b = L.gpu_alloc(ctx, arr.nbytes, 0)
            L.gpu_copy_to_device(ctx, b, arr.ctypes.data, arr.nbytes)
            bufs.append(b)
        C = L.gpu_alloc(ctx, M * N * 4, 0)
        L.gpu_matmul(ctx, C, bufs[0], bufs[1], M, N, K, 0, q)
        assert L.gpu_last_error(ctx) == 0
        got = np.empty((M, N), np.float32)
        L.gpu_copy_to_host(ctx, got.ctypes.data, C, got.nbytes)
        want = ref_matmul(oracle, A, oracle.dequant(blocks, wt, K * N).reshape(K, N))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    L.gpu_destroy(ctx)


@pytest.mark.parametrize("nbytes,off", [(8192, 0), (8190, 0), (4096, 3), (1 << 20, 0)])
def test_copy_kernel_host_and_device(ofb, cuda, nbytes, off):
    # ofb_copy between pinned host memory and the device, both directions,
    # aligned (16-byte path) and unaligned (byte path)
    src = torch.randint(0, 256, (nbytes + off,), dtype=torch.uint8).pin_memory()
    dev = torch.empty(nbytes + off, dtype=torch.uint8, device=cuda)
    back = torch.zeros(nbytes + off, dtype=torch.uint8).pin_memory()
    ofb._check(ofb.lib.ofb_copy(dev.data_ptr() + off, src.data_ptr() + off, nbytes, ofb._stream()))
    ofb._check(ofb.lib.ofb_copy(back.data_ptr() + off, dev.data_ptr() + off, nbytes, ofb._stream()))
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu()[off:], src[off:])
    assert torch.equal(back[off:], src[off:])
