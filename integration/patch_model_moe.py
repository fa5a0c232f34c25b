"""Writes a copy of the reference's engine/src/model.c whose routed-expert
block (inside model_forward's MoE FFN) calls the CUDA backend's
gpu_moe_forward through ofb_engine_moe_routed (engine_moe_cuda.c) instead of
decoding expert slices on the CPU. Everything else in the file is unchanged.
The edit is located by two comment lines of the block; it fails loudly if
they are not found, so a changed upstream file is noticed.

usage: python patch_model_moe.py <reference model.c> <output model.c>
"""
import sys

START = "if (lc->ffn_gate_inp) {"
END = "// Residual (via GPU if available)"
ANCHOR = "// ── Routed experts (top-k MoE)"


def main(src, dst):
    text = open(src).read()
    a = text.index(ANCHOR)
    s = text.index(START, a)
    e = text.index(END, s)
    line_start = text.rindex("\n", 0, e) + 1
    indent = " " * (e - line_start)
    repl = (START + "\n"
            f"{indent}/* routed experts on the GPU: gpu_moe_forward (renorm 0, ungated, interleaved slices) */\n"
            f"{indent}float *routed_out = (float *)alloca((size_t)D * sizeof(float));\n"
            f"{indent}ofb_engine_moe_routed(gpu, gguf, cfg, l, lc->ffn_gate_inp, ffn_x, routed_out);\n\n"
            f"{indent}")
    out = text[:s] + repl + text[e:]
    inc = '#include "memory.h"\n'
    out = out.replace(inc, inc + '#include "engine_moe_cuda.h"\n', 1)
    open(dst, "w").write(out)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
