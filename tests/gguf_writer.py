"""Minimal GGUF (version 3) writer for the loader tests: metadata scalars
(u32, f32, string) plus an array entry, and tensors with raw bytes, data
aligned to general.alignment. Test infrastructure only."""
import struct

import numpy as np

T_U32, T_F32, T_STR, T_ARR = 4, 6, 8, 9


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, arch, params, tensors, alignment=32):
    """params: {key: (type, value)} written with the architecture prefix
    unless the key starts with 'general.'; tensors: [(name, dims fastest
    first, ggml type, bytes)]."""
    meta = [("general.architecture", T_STR, arch), ("general.alignment", T_U32, alignment),
            ("general.tags", T_ARR, ["moe", "test"])]
    for k, (t, v) in params.items():
        meta.append((k if k.startswith("general.") else f"{arch}.{k}", t, v))
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, t, v in meta:
        out += _str(k) + struct.pack("<I", t)
        if t == T_U32:
            out += struct.pack("<I", v)
        elif t == T_F32:
            out += struct.pack("<f", v)
        elif t == T_STR:
            out += _str(v)
        elif t == T_ARR:
            out += struct.pack("<IQ", T_STR, len(v)) + b"".join(_str(x) for x in v)
    offs, off = [], 0
    for name, dims, ty, data in tensors:
        offs.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    for (name, dims, ty, data), o in zip(tensors, offs):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", ty, o)
    out += b"\0" * ((-len(out)) % alignment)
    for (name, dims, ty, data), o in zip(tensors, offs):
        out += bytes(data) + b"\0" * ((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(out)


def moe_layer_gguf(path, binding, d_model, hidden, n_experts, top_k, seed, layer=0, layout=0):
    """A one-layer file holding a seeded synthetic MoE layer (the bytes of
    binding.make_layer_host). layout 0 stores ggml's native order (router
    [E][D]); layout 1 the reference's reading (router [D][E])."""
    w = binding.make_layer_host(d_model, hidden, n_experts, layout=layout, seed=seed)
    D, H, E = d_model, hidden, n_experts
    b = f"blk.{layer}."
    tensors = [(b + "ffn_gate_inp.weight", [E, D] if layout == 1 else [D, E], 0, w["router"].tobytes()),
               (b + "ffn_gate_exps.weight", [D, H, E], 12, w["gate_exps"].tobytes()),
               (b + "ffn_up_exps.weight", [D, H, E], 12, w["up_exps"].tobytes()),
               (b + "ffn_down_exps.weight", [H, D, E], 14, w["down_exps"].tobytes()),
               (b + "ffn_gate_shexp.weight", [D, H], 12, w["gate_shexp"].tobytes()),
               (b + "ffn_up_shexp.weight", [D, H], 12, w["up_shexp"].tobytes()),
               (b + "ffn_down_shexp.weight", [H, D], 14, w["down_shexp"].tobytes()),
               (b + "ffn_gate_inp_shexp.weight", [D], 0, w["shexp_gate"].tobytes())]
    params = {"embedding_length": (T_U32, D), "expert_feed_forward_length": (T_U32, H),
              "expert_count": (T_U32, E), "expert_used_count": (T_U32, top_k), "block_count": (T_U32, 1),
              "rope.freq_base": (T_F32, 10000.0)}
    write_gguf(path, "ornith", params, tensors)
    return w


def engine_model_gguf(path, binding, d_model=256, hidden=256, n_experts=8, top_k=2, seed=1):
    """A one-layer model the reference engine's model_load / model_forward
    accept: attention weights zero (the attention adds nothing), norm weights
    one, output.weight the identity (vocab = d_model), so the logits are
    x + MoE(rmsnorm(x)) for x = the token's embedding row. MoE tensors in the
    reference's reading (router [D][E], expert index fastest) with the bytes
    of binding.make_layer_host(layout=1)."""
    D, H, E, V = d_model, hidden, n_experts, d_model
    nh, nkv = 2, 1
    w = binding.make_layer_host(D, H, E, layout=1, seed=seed)
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32).tobytes()
    emb = np.random.default_rng(seed).normal(size=(D, V)).astype(np.float32)
    b = "blk.0."
    tensors = [("token_embd.weight", [V, D], 0, f32(emb)),
               (b + "attn_norm.weight", [D], 0, f32(np.ones(D))),
               (b + "attn_q.weight", [nh * D, D], 0, f32(np.zeros(D * nh * D))),
               (b + "attn_k.weight", [nkv * 2, D], 0, f32(np.zeros(D * nkv * 2))),
               (b + "attn_v.weight", [nkv * 2, D], 0, f32(np.zeros(D * nkv * 2))),
               (b + "attn_output.weight", [D, nh * 2], 0, f32(np.zeros(nh * 2 * D))),
               (b + "post_attention_norm.weight", [D], 0, f32(np.ones(D))),
               (b + "ffn_gate_shexp.weight", [H, D], 12, w["gate_shexp"].tobytes()),
               (b + "ffn_up_shexp.weight", [H, D], 12, w["up_shexp"].tobytes()),
               (b + "ffn_down_shexp.weight", [D, H], 14, w["down_shexp"].tobytes()),
               (b + "ffn_gate_inp.weight", [E, D], 0, w["router"].tobytes()),
               (b + "ffn_gate_exps.weight", [D, H, E], 12, w["gate_exps"].tobytes()),
               (b + "ffn_up_exps.weight", [D, H, E], 12, w["up_exps"].tobytes()),
               (b + "ffn_down_exps.weight", [H, D, E], 14, w["down_exps"].tobytes()),
               ("output.weight", [V, D], 0, f32(np.eye(D)))]
    params = {"block_count": (T_U32, 1), "embedding_length": (T_U32, D), "attention.head_count": (T_U32, nh),
              "attention.head_count_kv": (T_U32, nkv), "expert_count": (T_U32, E),
              "expert_used_count": (T_U32, top_k), "feed_forward_length": (T_U32, H),
              "expert_feed_forward_length": (T_U32, H), "context_length": (T_U32, 64),
              "vocab_size": (T_U32, V), "attention.key_length": (T_U32, 2),
              "attention.value_length": (T_U32, 2), "rope.dimension_count": (T_U32, 2),
              "rope.freq_base": (T_F32, 10000.0), "full_attention_interval": (T_U32, 1)}
    write_gguf(path, "qwen2moe", params, tensors)
    return w, emb
