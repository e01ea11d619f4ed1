"""Seeded synthetic checkpoints and prompts (no network: no real weights or tokenizer).

Recipe (frozen; tests, golden fixtures and the benchmark all use it):
  * every parameter with ndim >= 2 (embeddings, linears, conv1d) ~ N(0, 0.02), drawn from a
    torch.Generator seeded with (seed, crc32(name)) so each tensor is reproducible on its own;
  * 1-D parameters take the HF constructor defaults: Qwen3RMSNorm = 1, Qwen3_5RMSNorm = 0
    (the (1 + w) form), gated norm = 1, dt_bias = 1, A_log = log(U(1, 16));
  * ``jitter > 0`` adds N(0, jitter) to norm weights and dt_bias so that parity tests exercise
    non-trivial per-channel scales;
  * weights are cast to bf16 (the reference's export dtype, compiler/qwen35/model.py:34-35).
Names follow HF Qwen3ForCausalLM / Qwen3_5ForCausalLM; lm_head is tied to embed_tokens.
"""

import zlib

import torch

from .configs import QWEN35


def _gen(seed, name, device):
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
    return g


def parameter_shapes(geometry):
    """Ordered {name: (shape, kind)} of the text model's parameters."""
    g = geometry
    H, I = g.hidden, g.intermediate
    shapes = {"model.embed_tokens.weight": ((g.vocab, H), "linear")}
    q35 = g.family == QWEN35
    norm_kind = "norm0" if q35 else "norm1"
    for i in range(g.num_layers):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = ((H,), norm_kind)
        if g.is_delta(i):
            key, val = g.lin_key_heads * g.lin_head_dim, g.lin_value_heads * g.lin_head_dim
            a = p + "linear_attn."
            shapes[a + "in_proj_qkv.weight"] = ((2 * key + val, H), "linear")
            shapes[a + "in_proj_z.weight"] = ((val, H), "linear")
            shapes[a + "in_proj_b.weight"] = ((g.lin_value_heads, H), "linear")
            shapes[a + "in_proj_a.weight"] = ((g.lin_value_heads, H), "linear")
            shapes[a + "conv1d.weight"] = ((g.conv_channels, 1, g.conv_width), "linear")
            shapes[a + "dt_bias"] = ((g.lin_value_heads,), "dt_bias")
            shapes[a + "A_log"] = ((g.lin_value_heads,), "a_log")
            shapes[a + "norm.weight"] = ((g.lin_head_dim,), "norm1")
            shapes[a + "out_proj.weight"] = ((H, val), "linear")
        else:
            a = p + "self_attn."
            shapes[a + "q_proj.weight"] = ((g.q_rows, H), "linear")
            shapes[a + "k_proj.weight"] = ((g.num_kv_heads * g.head_dim, H), "linear")
            shapes[a + "v_proj.weight"] = ((g.num_kv_heads * g.head_dim, H), "linear")
            shapes[a + "o_proj.weight"] = ((H, g.num_q_heads * g.head_dim), "linear")
            shapes[a + "q_norm.weight"] = ((g.head_dim,), norm_kind)
            shapes[a + "k_norm.weight"] = ((g.head_dim,), norm_kind)
        shapes[p + "post_attention_layernorm.weight"] = ((H,), norm_kind)
        shapes[p + "mlp.gate_proj.weight"] = ((I, H), "linear")
        shapes[p + "mlp.up_proj.weight"] = ((I, H), "linear")
        shapes[p + "mlp.down_proj.weight"] = ((H, I), "linear")
    shapes["model.norm.weight"] = ((H,), norm_kind)
    return shapes


def make_tensor(name, shape, kind, *, seed=0, jitter=0.0, device="cpu", dtype=torch.bfloat16):
    gen = _gen(seed, name, device)
    if kind == "linear":
        t = torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, 0.02, generator=gen)
    elif kind == "a_log":
        t = torch.empty(shape, device=device, dtype=torch.float32).uniform_(1.0, 16.0, generator=gen).log()
    else:
        base = {"norm0": 0.0, "norm1": 1.0, "dt_bias": 1.0}[kind]
        t = torch.full(shape, base, device=device, dtype=torch.float32)
        if jitter:
            t += torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, jitter, generator=gen)
    return t.to(dtype)


def make_state_dict(geometry, *, seed=0, jitter=0.0, device="cpu", dtype=torch.bfloat16):
    """HF-named state dict (tied lm_head shares embed_tokens storage)."""
    sd = {
        name: make_tensor(name, shape, kind, seed=seed, jitter=jitter, device=device, dtype=dtype)
        for name, (shape, kind) in parameter_shapes(geometry).items()
    }
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def random_prompt(geometry, length, *, seed=0):
    """Token IDs ~ U[0, vocab) (BASELINE's synthetic prompts)."""
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(0, geometry.vocab, (length,), generator=g).tolist()
