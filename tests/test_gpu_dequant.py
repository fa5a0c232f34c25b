"""Device dequant (ofb_dequantize / ofb_dequantize_expert_slice) bit-exact
against the reference's dequant: golden vectors from the reference's own
gguf.c, the oracle on seeded random blocks, and BASELINE config 5 sizes
(1 / 8 / 256 experts x 512 x 2048) in f32 and bf16."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = np.load(__file__.replace("test_gpu_dequant.py", "golden/dequant_golden.npz"))


def bf16_rne_bits(f32: np.ndarray) -> np.ndarray:
    return torch.from_numpy(f32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name,qtype", [("q4k", 12), ("q6k", 14)])
def test_golden_blocks(ofb, cuda, name, qtype):
    blocks = torch.from_numpy(GOLD[f"{name}_blocks"].reshape(-1)).to(cuda)
    n = GOLD[f"{name}_blocks"].shape[0] * 256
    got = ofb.dequantize(blocks, qtype, n).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, GOLD[f"{name}_values"])
    got16 = ofb.dequantize(blocks, qtype, n, out_dtype=torch.bfloat16).cpu().view(torch.int16).numpy()
    want16 = bf16_rne_bits(GOLD[f"{name}_values"].view(np.float32))
    assert np.array_equal(got16.view(np.uint16), want16)


@pytest.mark.parametrize("name,qtype", [("q4k", 12), ("q6k", 14)])
@pytest.mark.parametrize("ne", [4, 256])
def test_golden_slices(ofb, cuda, name, qtype, ne):
    blocks = torch.from_numpy(GOLD[f"{name}_slice{ne}_blocks"]).to(cuda)
    for e in range(ne):
        got = ofb.dequantize_slice(blocks, qtype, 256 * ne, ne, e).cpu().numpy().view(np.uint32)
        assert np.array_equal(got, GOLD[f"{name}_slice{ne}_values"][e]), e


@pytest.mark.parametrize("n_experts", [1, 8, 256])
@pytest.mark.parametrize("qtype", [12, 14])
def test_config5_sweep_vs_oracle(ofb, oracle, cuda, n_experts, qtype):
    nb = n_experts * 512 * 2048 // 256
    dev = ofb.synth_blocks(qtype, nb, seed=5, stream_id=qtype, device=cuda)
    n = nb * 256
    got = ofb.dequantize(dev, qtype, n).cpu().numpy()
    want = oracle.dequant(dev.cpu().numpy(), qtype, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    got16 = ofb.dequantize(dev, qtype, n, out_dtype=torch.bfloat16).cpu().view(torch.int16).numpy()
    assert np.array_equal(got16.view(np.uint16), bf16_rne_bits(want))


@pytest.mark.parametrize("qtype", [12, 14])
def test_ragged_block_counts(ofb, oracle, cuda, qtype):
    # Q6_K stages runs of 8 blocks; counts that are not multiples of 8 take the tail path
    for nb in (1, 7, 9, 15, 17):
        dev = ofb.synth_blocks(qtype, nb, seed=9, stream_id=nb, device=cuda)
        got = ofb.dequantize(dev, qtype, nb * 256).cpu().numpy()
        want = oracle.dequant(dev.cpu().numpy(), qtype, nb * 256)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), nb


def test_device_generator_matches_host(ofb, cuda):
    for qtype in (12, 14):
        d = ofb.synth_blocks(qtype, 333, seed=3, stream_id=4, device=cuda, first_block=10).cpu()
        h = ofb.synth_blocks_host(qtype, 333, seed=3, stream_id=4, first_block=10)
        assert torch.equal(d, h)


def test_slice_argument_checks(ofb, cuda):
    blocks = torch.zeros(144, dtype=torch.uint8, device=cuda)
    for e in (-1, 4, 99):
        with pytest.raises(ofb.OfbError) as ei:
            ofb.dequantize_slice(blocks, 12, 256, 4, e)
        assert ei.value.status == ofb.EINVAL
    with pytest.raises(ofb.OfbError):
        ofb.dequantize(blocks, 2, 256)  # Q4_0: not a type of this path


def test_empty_input_is_a_noop(ofb, cuda):
    blocks = torch.zeros(16, dtype=torch.uint8, device=cuda)
    out = torch.full((8,), 7.0, device=cuda)
    ofb.dequantize(blocks, 12, 0, out=out)
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)


def test_f16_every_bit_pattern(ofb, oracle, cuda):
    # gguf_dequantize_tensor_from_buf's F16 branch (engine/src/gguf.c:605-638)
    # uses the reference's non-IEEE fp16 rule (gguf.c:16-26): only 0x0000 maps
    # to zero; -0, subnormals and exponent-31 patterns decode as if normal.
    # All 65,536 patterns, as f32 bits and as bf16 (RNE of the f32 value).
    pats = np.arange(65536, dtype=np.uint16)
    dev = torch.from_numpy(pats.view(np.uint8).copy()).to(cuda)
    got = ofb.dequantize(dev, ofb.TYPE_F16, 65536).cpu().numpy()
    want = oracle.dequant(pats.view(np.uint8), ofb.TYPE_F16, 65536)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for p in (0x8000, 0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7FFF):  # the rebias edge cases
        assert np.isfinite(want[p]) and want[p] != 0.0, hex(p)
    got16 = ofb.dequantize(dev, ofb.TYPE_F16, 65536, out_dtype=torch.bfloat16).cpu().view(torch.int16).numpy()
    assert np.array_equal(got16.view(np.uint16), bf16_rne_bits(want))


def test_f32_copies_bits(ofb, oracle, cuda):
    # F32 branch: a bit copy (NaN payloads, infinities and -0 included); to
    # bf16 it rounds to nearest even like torch (checked on finite values)
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2**32, size=4096, dtype=np.uint64).astype(np.uint32)
    bits[:6] = [0x80000000, 0x7F800000, 0xFF800000, 0x7FC00001, 0x00000001, 0x3F800000]
    dev = torch.from_numpy(bits.view(np.uint8).copy()).to(cuda)
    got = ofb.dequantize(dev, ofb.TYPE_F32, 4096).cpu().numpy()
    want = oracle.dequant(bits.view(np.uint8), ofb.TYPE_F32, 4096)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    finite = np.isfinite(want)
    got16 = ofb.dequantize(dev, ofb.TYPE_F32, 4096, out_dtype=torch.bfloat16).cpu().view(torch.int16).numpy()
    assert np.array_equal(got16.view(np.uint16)[finite], bf16_rne_bits(want)[finite])


@pytest.mark.parametrize("qtype", [0, 1])
def test_plain_type_slices(ofb, oracle, cuda, qtype):
    # expert slices of F32 / F16 tensors (gguf.c:652-711 handles every type)
    ne, per = 5, 300
    rng = np.random.default_rng(qtype)
    if qtype == 0:
        raw = rng.normal(size=ne * per).astype(np.float32).view(np.uint8)
    else:
        raw = rng.integers(0, 65536, size=ne * per, dtype=np.uint32).astype(np.uint16).view(np.uint8)
    dev = torch.from_numpy(raw.copy()).to(cuda)
    for e in range(ne):
        got = ofb.dequantize_slice(dev, qtype, ne * per, ne, e).cpu().numpy()
        want = oracle.dequant_slice(raw, qtype, ne * per, ne, e)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), e
