"""Generate tests/golden/dequant_golden.npz from the reference itself.

Runs the reference's own engine/src/gguf.c (compiled unmodified into
oracle/_ref/libref.so by `make -C oracle`) on seeded random Q4_K / Q6_K
blocks, including the fp16 scale patterns its non-IEEE decode treats
specially (0x0000, 0x8000 = -0, subnormals, exponent 31, NaN/inf patterns),
and on expert-slice tensors. The committed .npz pins the oracle and the CUDA
kernels without needing the reference tree at test time.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import binding  # noqa: E402

SPECIAL_HALF = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x7C00, 0x7E00, 0xFC00,
                0xFFFF, 0x8001, 0x83FF, 0x2E66, 0x211F, 0x0200]


def random_blocks(rng, n, nbytes, scale_offsets):
    b = rng.integers(0, 256, size=(n, nbytes), dtype=np.uint8)
    # d/dmin: mostly realistic U(0, 0.01) fp16, some special bit patterns
    for off in scale_offsets:
        vals = np.float16(rng.uniform(0, 0.01, size=n)).view(np.uint16).copy()
        sp = rng.integers(0, len(SPECIAL_HALF), size=n)
        use_sp = rng.random(n) < 0.3
        vals[use_sp] = np.array(SPECIAL_HALF, dtype=np.uint16)[sp[use_sp]]
        b[:, off] = (vals & 0xFF).astype(np.uint8)
        b[:, off + 1] = (vals >> 8).astype(np.uint8)
    return b


def main():
    ref = binding.load_ref()
    if ref is None:
        sys.exit("oracle/_ref/libref.so missing: run `make -C oracle` with the reference tree present")
    rng = np.random.default_rng(20261201)
    out = {}
    for name, qtype, nbytes, offs in (("q4k", binding.TYPE_Q4_K, 144, (0, 2)),
                                       ("q6k", binding.TYPE_Q6_K, 210, (208,))):
        blocks = random_blocks(rng, 96, nbytes, offs)
        vals = binding.dequant(blocks.reshape(-1), qtype, 96 * 256, lib=ref)
        out[f"{name}_blocks"] = blocks
        out[f"{name}_values"] = vals.view(np.uint32)
        # expert slices: n_experts 4 (the reference test's shape) and 256
        for ne in (4, 256):
            nelem = 256 * ne  # one block per expert-row group
            sb = random_blocks(rng, nelem // 256, nbytes, offs).reshape(-1)
            sl = np.stack([binding.dequant_slice(sb, qtype, nelem, ne, e, lib=ref) for e in range(ne)])
            out[f"{name}_slice{ne}_blocks"] = sb
            out[f"{name}_slice{ne}_values"] = sl.view(np.uint32)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
