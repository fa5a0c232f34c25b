"""Host side of the seeded generator (the device kernel must produce the same
bytes: tests/test_gpu_dequant.py::test_device_generator_matches_host)."""
import numpy as np


def test_blocks_deterministic_and_scaled(ofb, oracle):
    a = ofb.synth_blocks_host(ofb.TYPE_Q4_K, 64, seed=5, stream_id=1).numpy()
    b = ofb.synth_blocks_host(ofb.TYPE_Q4_K, 64, seed=5, stream_id=1).numpy()
    c = ofb.synth_blocks_host(ofb.TYPE_Q4_K, 64, seed=6, stream_id=1).numpy()
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    blk = a.reshape(64, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float64).ravel()
    assert np.all((d >= 0) & (d <= 0.01)) and np.all((dmin >= 0) & (dmin <= 0.01))
    # d is RNE(U(0,0.01)) in fp16: the 6-bit scales are uniform
    assert len(np.unique(blk[:, 4:16])) > 200


def test_first_block_offset(ofb):
    whole = ofb.synth_blocks_host(ofb.TYPE_Q6_K, 20, seed=1, stream_id=3).numpy()
    tail = ofb.synth_blocks_host(ofb.TYPE_Q6_K, 5, seed=1, stream_id=3, first_block=15).numpy()
    assert np.array_equal(whole[15 * 210:], tail)
    d = whole.reshape(20, 210)[:, 208:210].copy().view(np.float16).astype(np.float64)
    assert np.all((d >= 0) & (d <= 0.01))


def test_normal_moments(ofb):
    x = ofb.synth_normal(200000, seed=0, stream_id=9, sigma=0.02).numpy()
    assert abs(x.mean()) < 2e-4 and abs(x.std() - 0.02) < 2e-4


def test_oracle_generator_matches_library(ofb, oracle):
    # the CPU legs of the benchmark build layers with the oracle's copy of the
    # generator (no product library loaded there): it must give the same bytes
    for q, n in ((ofb.TYPE_Q4_K, 37), (ofb.TYPE_Q6_K, 41)):
        for first in (0, 1000):
            a = ofb.synth_blocks_host(q, n, seed=3, stream_id=q, first_block=first).numpy()
            b = oracle.synth_blocks(q, n, seed=3, stream_id=q, first_block=first)
            assert np.array_equal(a, b)
    a = ofb.synth_normal(10001, seed=4, stream_id=9, sigma=0.02).numpy()
    b = oracle.synth_normal(10001, seed=4, stream_id=9, sigma=0.02)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_layer_matches_library_layer(ofb, oracle):
    for layout in (0, 1):
        shape = ofb.LayerShape(d_model=512, hidden=256, n_experts=16, top_k=4, layout=layout)
        lw = ofb.make_layer(shape, seed=7, device="cpu")
        hw = oracle.make_layer_host(512, 256, 16, layout=layout, seed=7)
        for k, v in vars(lw).items():
            assert np.array_equal(v.numpy().view(np.uint8), hw[k].view(np.uint8)), k
    x = ofb.make_tokens(ofb.LayerShape(), 3, seed=5).numpy()
    assert np.array_equal(x, oracle.make_tokens_host(2048, 3, seed=5))
