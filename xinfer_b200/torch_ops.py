"""Torch custom operators (xinfer_b200/csrc/torch_ops.cpp, built into
xinfer_b200/libxinfer_b200_ops.so) with the fake kernels that torch.export / AOTInductor trace:
the decode step, xinfer::qwen35_decode_step and xinfer::qwen3_decode_step, and the reference's
attention operators xinfer::flash_attention and xinfer::batched_flash_attention
(compiler/common/kernels/attention.cpp:128-140) backed by this library's sm_100a attention kernel
instead of ATen's FlashAttention-2, so the library can stand in for libxinfer_attention_ops.so.

The operators keep ModelStep.forward's T == 1 contract (compiler/qwen35/model.py:162-183,
compiler/qwen3/model.py:70-95) and carry the model as arguments, the way an exported graph
carries its constants: `weights` in the order of weight_list(), `geometry` and `params` from
geometry_args(). The fake kernels mirror the reference's registration of its attention operators
(compiler/common/attention.py:47-96): shape checks with torch._check and outputs built from the
inputs' metadata only.

    from xinfer_b200 import torch_ops
    torch_ops.load()
    step = torch_ops.DecodeStep(geometry, weights, capacity)
    logits, *state = step(input_ids, cache_position, state, kv_lengths, query_lengths)
"""

from pathlib import Path

import torch

from .configs import QWEN35

LIBRARY = Path(__file__).resolve().parent / "libxinfer_b200_ops.so"
FAMILY = {"qwen3": 1, QWEN35: 2}
_loaded = False


def geometry_args(g, capacity, state_rows=8):
    """(geometry, params) operator arguments: XbGeometry's integer fields, one layer kind per
    layer (0 attention, 1 DeltaNet), then (rms_eps, rope_theta)."""
    ints = [FAMILY[g.family], g.num_layers, g.hidden, g.intermediate, g.vocab, g.num_q_heads,
            g.num_kv_heads, g.head_dim, g.rotary_dim, g.lin_key_heads, g.lin_value_heads,
            g.lin_head_dim, g.conv_width, int(capacity), int(state_rows)]
    ints += [1 if g.is_delta(i) else 0 for i in range(g.num_layers)]
    return ints, [float(g.rms_eps), float(g.rope_theta)]


def weight_list(g, weights):
    """The operator's weight tensors in order, from an HF-named state dict."""
    W = weights
    out = [W["model.embed_tokens.weight"], W["model.norm.weight"],
           W.get("lm_head.weight", W["model.embed_tokens.weight"])]
    for i in range(g.num_layers):
        p = f"model.layers.{i}."
        out += [W[p + "input_layernorm.weight"], W[p + "post_attention_layernorm.weight"],
                W[p + "mlp.gate_proj.weight"], W[p + "mlp.up_proj.weight"], W[p + "mlp.down_proj.weight"]]
        if g.is_delta(i):
            a = p + "linear_attn."
            out += [W[a + n] for n in ("in_proj_qkv.weight", "in_proj_z.weight", "in_proj_b.weight",
                                       "in_proj_a.weight", "conv1d.weight", "A_log", "dt_bias",
                                       "norm.weight", "out_proj.weight")]
        else:
            a = p + "self_attn."
            out += [W[a + n] for n in ("q_proj.weight", "k_proj.weight", "v_proj.weight",
                                       "o_proj.weight", "q_norm.weight", "k_norm.weight")]
    return out


def _check_inputs(input_ids, cache_position, state, kv_lengths, query_lengths, geometry):
    torch._check(input_ids.dim() == 2 and input_ids.shape[1] == 1)
    torch._check(input_ids.dtype == torch.int64 and input_ids.device.type == "cuda")
    torch._check(cache_position.shape == input_ids.shape and cache_position.dtype == torch.int64)
    torch._check(kv_lengths.device.type == "cpu" and kv_lengths.dtype == torch.int32)
    torch._check(query_lengths.device.type == "cpu" and query_lengths.dtype == torch.int32)
    torch._check(kv_lengths.shape == (input_ids.shape[0],) and query_lengths.shape == kv_lengths.shape)
    torch._check(1 <= input_ids.shape[0] <= 8)
    torch._check(len(geometry) == 15 + geometry[1])
    torch._check(len(state) == 2 * geometry[1])


def _fake_outputs(input_ids, state, geometry):
    batch, vocab, layers = input_ids.shape[0], geometry[4], geometry[1]
    out = [input_ids.new_empty((batch, vocab), dtype=torch.bfloat16)]
    for i in range(layers):
        if geometry[15 + i] == 1:
            out += [torch.empty_like(state[2 * i]), torch.empty_like(state[2 * i + 1])]
    return out


def load(library=None):
    """Load the operator library once and register its fake kernels."""
    global _loaded
    if _loaded:
        return
    path = Path(library or LIBRARY)
    if not path.is_file():
        raise FileNotFoundError(f"{path} is missing: build it with `python -m xinfer_b200.build`")
    torch.ops.load_library(str(path))

    @torch.library.register_fake("xinfer::qwen35_decode_step")
    def fake35(input_ids, cache_position, state, kv_lengths, query_lengths, weights, geometry, params):
        torch._check(geometry[0] == FAMILY[QWEN35])
        _check_inputs(input_ids, cache_position, state, kv_lengths, query_lengths, geometry)
        return _fake_outputs(input_ids, state, geometry)

    @torch.library.register_fake("xinfer::qwen3_decode_step")
    def fake3(input_ids, cache_position, state, kv_lengths, query_lengths, weights, geometry, params):
        torch._check(geometry[0] == FAMILY["qwen3"])
        _check_inputs(input_ids, cache_position, state, kv_lengths, query_lengths, geometry)
        return _fake_outputs(input_ids, state, geometry)[0]

    @torch.library.register_fake("xinfer::flash_attention")
    def fake_attention(q, k, v, kv_extent, scale):
        # as the reference's registration (compiler/common/attention.py:63-82): output
        # metadata depends on Q only; the valid-prefix length is checked natively
        torch._check(q.dim() == 4 and k.dim() == 4 and v.dim() == 4)
        torch._check(q.shape[0] > 0 and q.shape[1] > 0 and k.shape[1] > 0)
        torch._check(q.shape[1] % k.shape[1] == 0)
        torch._check(q.shape[3] >= 8 and q.shape[3] <= 256 and q.shape[3] % 8 == 0)
        torch._check(q.shape[2] >= 1 and q.shape[2] <= 512 and k.shape[2] > 0)
        torch._check(k.shape == (q.shape[0], k.shape[1], k.shape[2], q.shape[3]) and v.shape == k.shape)
        torch._check(q.dtype == k.dtype == v.dtype == torch.bfloat16)
        torch._check(q.device.type == "cuda" and k.device == q.device and v.device == q.device)
        torch._check(kv_extent.device.type == "cpu" and kv_extent.dtype == torch.uint8 and kv_extent.dim() == 1)
        return q.new_empty(q.shape)

    @torch.library.register_fake("xinfer::batched_flash_attention")
    def fake_batched(q, k, v, offsets, cuda_offsets, blocks, scale):
        torch._check(offsets.device.type == "cpu" and offsets.dtype == torch.int32)
        torch._check(offsets.shape == (2, q.shape[0] + 1))
        torch._check(cuda_offsets.shape == offsets.shape and cuda_offsets.device == q.device)
        torch._check(blocks.shape == (q.shape[0], 1) and blocks.device == q.device)
        return fake_attention(q, k, v, torch.empty(2, dtype=torch.uint8), scale)

    _loaded = True


class DecodeStep(torch.nn.Module):
    """ModelStep.forward at T == 1 through the custom operator: returns (logits, *state) for
    Qwen3.5, whose conv / recurrent entries are fresh tensors and whose KV entries are the
    inputs (appended in place), and logits for Qwen3."""

    def __init__(self, geometry, weights, capacity, state_rows=8):
        super().__init__()
        load()
        self.g = geometry
        self.weights = weight_list(geometry, weights)
        self.geometry, self.params = geometry_args(geometry, capacity, state_rows)

    def forward(self, input_ids, cache_position, state, kv_lengths, query_lengths):
        args = (input_ids, cache_position, list(state), kv_lengths, query_lengths, self.weights,
                self.geometry, self.params)
        if self.g.family != QWEN35:
            return torch.ops.xinfer.qwen3_decode_step(*args)
        logits, *fresh = torch.ops.xinfer.qwen35_decode_step(*args)
        out, k = list(state), 0
        for i in range(self.g.num_layers):
            if self.g.is_delta(i):
                out[2 * i], out[2 * i + 1] = fresh[k], fresh[k + 1]
                k += 2
        return (logits, *out)
