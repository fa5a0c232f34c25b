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
