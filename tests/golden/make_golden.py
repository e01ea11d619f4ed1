"""Generate golden fixtures by running the reference's own decode step on the CPU.

Usage (needs a checkout of tqxia/xinfer; the fixtures are committed, so tests never run this):

    python tests/golden/make_golden.py --reference <path to the xinfer checkout> [--only NAME]

What runs is the reference's code, imported from the checkout, unmodified:
  * ModelStep / HybridCache / KVCache / text_rotary   (compiler/qwen35/model.py, compiler/qwen3/model.py)
  * the attention adapters and DeltaNet adapter       (compiler/qwen35/adapters/*, compiler/qwen3/adapters/*)
  * the Triton kernels fused_kernel (DeltaNet recurrence, recurrent.py:61-124) and _append (KV
    append, kv_cache.py:8-42), launched directly under Triton's CPU interpreter
    (TRITON_INTERPRET=1) with the same arguments their torch.library wrappers pass;
  * the HF transformers modules the adapters keep.
Three things are substituted because they need a GPU or the export toolchain:
  * xinfer::batched_flash_attention (ATen FlashAttention-2, attention.cpp:14-79) is registered
    here with a CPU implementation of the same contract: per-row valid prefix, lower-right
    causal, GQA without expansion, zero rows for empty queries; probabilities rounded to bf16
    before the P.V product as FlashAttention-2 does;
  * libdevice.exp / log1p inside recurrent.py become tl.exp and an accurate log1p
    (log1p(x) = log(u) * x / (u - 1), u = 1 + x);
  * the interpreter's fp32 -> bf16 cast (which truncates) is replaced by round-to-nearest-even,
    the rounding the GPU's cvt.rn.bf16.f32 performs.
The Qwen3 ModelStep was written against transformers 4.51 (decoder layers returning tuples,
a Cache base class constructible without arguments); under the installed 5.x each decoder
layer is wrapped to return a one-tuple and Cache() without arguments is allowed again.

Weights: the seeded synthetic recipe of xinfer_b200/synthetic.py (norm jitter 0.1 so norms are
non-trivial). Fixtures store inputs, per-step logits and (sampled) state.
"""

import argparse
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from xinfer_b200 import configs, synthetic  # noqa: E402

HERE = Path(__file__).resolve().parent
SAMPLES = 4096


@triton.jit
def _exp(x):
    return tl.exp(x)


@triton.jit
def _log1p(x):
    u = 1.0 + x
    return tl.where(u == 1.0, x, tl.log(u) * (x / (u - 1.0)))


def patch_interpreter_rounding():
    from triton.runtime import interpreter as TI

    orig_cast = TI.InterpreterBuilder.cast_impl
    orig_fp = TI.InterpreterBuilder.create_fp_to_fp

    def rtne(src):
        f = torch.from_numpy(np.ascontiguousarray(src.data).astype(np.float32))
        return f.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return TI.TensorHandle(rtne(src), dst_type.scalar)
        return orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return TI.TensorHandle(rtne(src), dst_type.scalar)
        return orig_fp(self, src, dst_type, rounding_mode)

    TI.InterpreterBuilder.cast_impl = cast_impl
    TI.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp


def register_cpu_attention():
    """CPU stand-in for xinfer::batched_flash_attention with the contract of attention.cpp:14-79."""
    lib = torch.library.Library("xinfer", "DEF")
    lib.define("batched_flash_attention(Tensor q, Tensor k, Tensor v, Tensor offsets, "
               "Tensor cuda_offsets, Tensor blocks, float scale) -> Tensor")

    def impl(q, k, v, offsets, cuda_offsets, blocks, scale):
        batch, hq, tq, d = q.shape
        hkv = k.shape[1]
        group = hq // hkv
        cuq, cuk = offsets[0].tolist(), offsets[1].tolist()
        out = torch.zeros_like(q)
        for row in range(batch):
            count, length = cuq[row + 1] - cuq[row], cuk[row + 1] - cuk[row]
            assert 0 <= count <= tq and length >= count and 1 <= length <= k.shape[2]
            if count == 0:
                continue
            qr = q[row, :, :count].float()
            kr = k[row, :, :length].float().repeat_interleave(group, 0)
            vr = v[row, :, :length].float().repeat_interleave(group, 0)
            s = torch.einsum("hqd,hkd->hqk", qr, kr) * scale
            qpos = torch.arange(count)[:, None] + (length - count)
            s = s.masked_fill(torch.arange(length)[None, :] > qpos, float("-inf"))
            m = s.amax(-1, keepdim=True)
            p = torch.exp(s - m)
            lsum = p.sum(-1, keepdim=True)
            o = torch.einsum("hqk,hkd->hqd", p.to(torch.bfloat16).float(), vr) / lsum
            out[row, :, :count] = o.to(q.dtype)
        return out

    lib.impl("batched_flash_attention", impl, "CPU")
    return lib


def import_reference(path):
    sys.path.insert(0, str(path))
    from compiler.qwen35.kernels import recurrent as R

    R.libdevice = types.SimpleNamespace(exp=_exp, log1p=_log1p)
    from compiler.common.kernels import kv_cache as KV

    def append_kv_batched(key, value, positions, cu_query, cache_key, cache_value):
        # the arguments of the reference's triton_op wrapper (kv_cache.py:45-72)
        assert cache_key.is_contiguous() and cache_value.is_contiguous()
        batch, heads, tokens, dim = key.shape
        KV._append[(triton.cdiv(tokens * dim, 256), heads, batch)](
            key, value, positions, cu_query, cache_key, cache_value, tokens, dim,
            cache_key.shape[2], heads, *key.stride(), *value.stride(), *positions.stride(), 256,
        )

    def fused(qkv, b, a, conv, state, weight, A_log, dt_bias, query_lengths=None):
        # the reference's dispatch (recurrent.py:292-349): chunks longer than SHORT_THRESHOLD
        # take its `long` path (prepare kernel + chunk-64 scan, recurrent.py:234-281), run as is
        batch, tokens = qkv.shape[:2]
        if query_lengths is None:
            query_lengths = torch.full((batch,), tokens, dtype=torch.int32)
        if tokens > R.SHORT_THRESHOLD:
            # wrap_triton (a pass-through outside torch.compile) rejects the interpreter's kernels
            wrap = torch.library.wrap_triton
            torch.library.wrap_triton = lambda kernel: kernel
            try:
                return R.long(qkv, b, a, conv, state, weight, A_log, dt_bias, query_lengths)
            finally:
                torch.library.wrap_triton = wrap
        # the arguments of the reference's `short` wrapper (recurrent.py:192-231)
        value_heads = state.shape[1]
        key_heads = (qkv.shape[2] // R.DIM - value_heads) // 2
        qkv, b, a, conv, weight, A_log, dt_bias, state = (
            x.contiguous() for x in (qkv, b, a, conv, weight, A_log, dt_bias, state))
        if query_lengths is None:
            query_lengths = torch.full((batch,), tokens, dtype=torch.int32)
        output = qkv.new_empty((batch, tokens, value_heads, R.DIM))
        next_conv, final = torch.empty_like(conv), torch.empty_like(state)
        R.fused_kernel[(value_heads, R.DIM // R.VALUE_TILE, batch)](
            qkv, b, a, conv, state, weight, A_log, dt_bias, output, next_conv, final,
            query_lengths.contiguous(), tokens, key_heads, value_heads, R.DIM, R.VALUE_TILE, 4,
            **R.OPTIONS,
        )
        return output, next_conv, final

    from transformers import cache_utils

    cache_init = cache_utils.Cache.__init__

    def permissive_cache_init(self, *args, **kwargs):
        if not args and not kwargs:
            self.layers = []
            return
        cache_init(self, *args, **kwargs)

    cache_utils.Cache.__init__ = permissive_cache_init

    import compiler.qwen35.model as M35
    import compiler.qwen3.model as M3
    import compiler.qwen35.adapters.attention as A35
    import compiler.qwen3.adapters.attention as A3
    import compiler.qwen35.adapters.delta as D35

    M35.append_kv_batched = append_kv_batched
    M3.append_kv_batched = append_kv_batched
    A35.load_attention_ops = lambda *args, **kwargs: None
    A3.load_attention_ops = lambda *args, **kwargs: None
    D35.fused = fused
    return types.SimpleNamespace(M35=M35, M3=M3, D35=D35)


class TupleLayer(torch.nn.Module):
    """transformers 5.x decoder layers return a tensor; the Qwen3 ModelStep indexes [0]."""

    def __init__(self, layer):
        super().__init__()
        self.layer = layer

    def forward(self, *args, **kwargs):
        return (self.layer(*args, **kwargs),)


def build_step(ref, geometry, sd):
    hf = configs.hf_config(geometry)
    hf._attn_implementation = "sdpa"
    if geometry.family == configs.QWEN35:
        from transformers import Qwen3_5ForCausalLM
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding

        with torch.device("meta"):
            model = Qwen3_5ForCausalLM(hf)
        model.load_state_dict(sd, strict=True, assign=True)
        model.lm_head.weight = model.model.embed_tokens.weight
        model.model.rotary_emb = Qwen3_5TextRotaryEmbedding(hf)
        model = model.eval().requires_grad_(False)
        ref.D35.install_delta(model)
        return ref.M35.ModelStep(model)
    from transformers import Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    with torch.device("meta"):
        model = Qwen3ForCausalLM(hf)
    model.load_state_dict(sd, strict=True, assign=True)
    model.lm_head.weight = model.model.embed_tokens.weight
    model.model.rotary_emb = Qwen3RotaryEmbedding(hf)
    model = model.eval().requires_grad_(False)
    step = ref.M3.ModelStep(model)
    step.model.model.layers = torch.nn.ModuleList(TupleLayer(layer) for layer in step.model.model.layers)
    return step


def zero_state(geometry, rows, capacity):
    out = []
    for i in range(geometry.num_layers):
        if geometry.is_delta(i):
            out.append(torch.zeros(rows, geometry.conv_channels, geometry.conv_width, dtype=torch.bfloat16))
            out.append(torch.zeros(rows, geometry.lin_value_heads, geometry.lin_head_dim,
                                   geometry.lin_head_dim))
        else:
            kv = (rows, geometry.num_kv_heads, capacity, geometry.head_dim)
            out.append(torch.zeros(kv, dtype=torch.bfloat16))
            out.append(torch.zeros(kv, dtype=torch.bfloat16))
    return out


@torch.inference_mode()
def run_schedule(step, geometry, state, schedule, capacity):
    """schedule: list of per-step row token lists ([] = empty row, several tokens = a prefill
    chunk of that row). Returns per-step logits (of each row's last token)."""
    rows = len(schedule[0])
    positions = [0] * rows
    logits_all = []
    for tokens in schedule:
        width = max(1, max(len(t) for t in tokens))
        ids = torch.tensor([list(t) + [0] * (width - len(t)) for t in tokens], dtype=torch.int64)
        pos = torch.tensor([[positions[r] + j for j in range(width)] for r in range(rows)], dtype=torch.int64)
        kv_lengths = torch.tensor([positions[r] + len(tokens[r]) for r in range(rows)], dtype=torch.int32)
        q_lengths = torch.tensor([len(t) for t in tokens], dtype=torch.int32)
        out = step(ids, pos, state, kv_lengths, q_lengths)
        if geometry.family == configs.QWEN35:
            logits, *fresh = out
            state = list(fresh)
        else:
            logits = out
        logits_all.append(logits.clone())
        for r in range(rows):
            positions[r] += len(tokens[r])
    return torch.stack(logits_all), state, positions


def sample_state(state, seed=1234):
    g = torch.Generator().manual_seed(seed)
    out = []
    for t in state:
        flat = t.reshape(-1)
        if flat.numel() <= SAMPLES:
            idx = torch.arange(flat.numel(), dtype=torch.int32)
        else:
            idx = torch.randint(0, flat.numel(), (SAMPLES,), generator=g, dtype=torch.int32)
        out.append({"index": idx, "value": flat[idx.long()].clone(), "sum": float(t.double().sum()),
                    "abs_sum": float(t.double().abs().sum()), "shape": tuple(t.shape)})
    return out


def make_schedules(geometry, kind, seed):
    g = torch.Generator().manual_seed(seed)
    tok = lambda: int(torch.randint(0, geometry.vocab, (1,), generator=g))  # noqa: E731
    if kind == "single":
        return [[[tok()]] for _ in range(10)]
    if kind == "batch":
        # three rows, ragged starts, empty rows in some steps (rows need history before empty)
        active = [
            (1, 1, 1), (1, 1, 0), (1, 0, 1), (0, 1, 1), (1, 1, 0), (1, 1, 1), (1, 0, 1), (0, 1, 1),
        ]
        return [[[tok()] if a else [] for a in row] for row in active]
    if kind == "short":
        return [[[tok()]] for _ in range(4)]
    if kind == "long16":
        return [[[tok()]] for _ in range(16)]
    if kind == "prefill128":
        # one 128-token prefill chunk (the reference's long DeltaNet path), then 4 decode steps
        return [[[tok() for _ in range(128)]]] + [[[tok()]] for _ in range(4)]
    raise ValueError(kind)


CASES = {
    # name: (config, schedule kind, capacity, jitter, full logits: True, False, or the number of
    # final steps whose full rows are stored)
    "qwen3-tiny-single": ("qwen3-tiny", "single", 16, 0.1, True),
    "qwen3-tiny-batch": ("qwen3-tiny", "batch", 16, 0.1, True),
    "qwen3.5-tiny-single": ("qwen3.5-tiny", "single", 16, 0.1, True),
    "qwen3.5-tiny-batch": ("qwen3.5-tiny", "batch", 16, 0.1, True),
    "qwen3.5-tiny-hv32-single": ("qwen3.5-tiny-hv32", "single", 16, 0.1, True),
    "qwen3.5-tiny-prefill128": ("qwen3.5-tiny", "prefill128", 256, 0.1, True),
    "qwen3-0.6b-short": ("qwen3-0.6b", "short", 16, 0.0, False),
    "qwen3.5-0.8b-short": ("qwen3.5-0.8b", "short", 16, 0.0, False),
    # the headline geometry at the headline KV capacity: full depth, 4096 slots, 16 steps, the
    # last 8 logits rows stored whole (one reference step takes about a minute on the CPU)
    "qwen3.5-0.8b-cap4096": ("qwen3.5-0.8b", "long16", 4096, 0.0, 8),
}


def summarize_logits(logits):
    flat = logits.float()
    top = flat.topk(32, dim=-1)
    return {"argmax": flat.argmax(-1), "top_values": top.values, "top_indices": top.indices,
            "stride_slice": logits[..., ::97].clone(), "sum": flat.double().sum(-1)}


def generate(ref, name, seed=0):
    config, kind, capacity, jitter, full = CASES[name]
    geometry = configs.get(config)
    sd = synthetic.make_state_dict(geometry, seed=seed, jitter=jitter)
    step = build_step(ref, geometry, sd)
    schedule = make_schedules(geometry, kind, seed=7)
    rows = len(schedule[0])
    state = zero_state(geometry, rows, capacity)
    logits, state, positions = run_schedule(step, geometry, state, schedule, capacity)
    fixture = {
        "name": name, "config": config, "seed": seed, "jitter": jitter, "capacity": capacity,
        "schedule": schedule, "positions": positions,
        "logits": logits if full is True else None,
        "logits_tail": logits[-full:].clone() if full is not True and full else None,
        "logits_summary": summarize_logits(logits),
        "state_sample": sample_state(state),
        "conv_state": [t.clone() for i, t in enumerate(state)
                       if geometry.is_delta(i // 2) and i % 2 == 0] if full is True else None,
    }
    out = HERE / f"{name}.pt"
    torch.save(fixture, out)
    print(f"wrote {out} ({out.stat().st_size / 1024:.0f} KiB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the tqxia/xinfer checkout")
    ap.add_argument("--only", action="append")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    patch_interpreter_rounding()
    library = register_cpu_attention()  # keep the registration alive
    ref = import_reference(Path(args.reference))
    for name in args.only or CASES:
        generate(ref, name)
    del library


if __name__ == "__main__":
    main()
