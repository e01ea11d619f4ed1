"""CPU oracle of the Qwen3 / Qwen3.5 decode step — TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA decode path. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it; the product path never does.

It restates, in fp32 torch on the CPU, the reference's decode step at T == 1 with the same
bf16 rounding points (each op's output tensor is bf16 in the reference, math inside an op is
fp32). Pinned against the reference itself: tests/golden/make_golden.py runs the reference's
own ModelStep (HF modules + xinfer adapters + xinfer's Triton DeltaNet/KV kernels under the
Triton CPU interpreter) and the CPU tests compare this oracle with those fixtures.

Reference citations (paths inside tqxia/xinfer):
  step loop, last-token gather, lm_head, masked_fill  compiler/qwen35/model.py:162-183,
                                                      compiler/qwen3/model.py:70-95
  Qwen3.5 attention adapter (query/gate split, norms, RoPE, sigmoid gate)
                                                      compiler/qwen35/adapters/attention.py:39-63
  Qwen3 attention adapter                             compiler/qwen3/adapters/attention.py:31-62
  text RoPE tables                                    compiler/qwen35/model.py:144-151
  KV append                                           compiler/common/kernels/kv_cache.py:8-42
  prefix attention (lower-right causal, GQA)          compiler/common/kernels/attention.cpp:14-79
  DeltaNet adapter (projections, gated norm)          compiler/qwen35/adapters/delta.py:32-49
  DeltaNet conv + recurrence                          compiler/qwen35/kernels/recurrent.py:20-124
HF modules the adapters keep (transformers): Qwen3RMSNorm, Qwen3_5RMSNorm, Qwen3_5RMSNormGated,
Qwen3MLP / Qwen3_5MLP, apply_rotary_pos_emb, rotate_half.
"""

import math

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def rbf(x):
    """Round an fp32 tensor through bf16 (a bf16 tensor boundary in the reference)."""
    return x.to(BF16).float()


def fma32(a, b, c):
    """fp32 fused multiply-add (Triton fuses `total += x * w` with fp fusion enabled)."""
    return (a.double() * b.double() + c.double()).float()


def prepare_weights(state_dict):
    """fp32 copies (exact bf16 values) of an HF-named bf16 state dict."""
    return {k: v.float() for k, v in state_dict.items()}


# Accumulation type of the linears. fp32 is the reference's (cuBLAS fp32 accumulation);
# fp64 gives the "twin" oracle whose difference from the fp32 one measures how far two valid
# summation orders drift apart on a given workload (the noise floor the GPU parity tests use).
_LINEAR_ACC = torch.float32


class accumulate(object):
    """Context manager: run the oracle's linears with another accumulation dtype."""

    def __init__(self, dtype):
        self.dtype = dtype

    def __enter__(self):
        global _LINEAR_ACC
        self.prev, _LINEAR_ACC = _LINEAR_ACC, self.dtype
        return self

    def __exit__(self, *exc):
        global _LINEAR_ACC
        _LINEAR_ACC = self.prev


def linear(x, w):
    """bf16 linear: fp32 accumulate, bf16 output (cuBLAS GEMM as lowered by Inductor)."""
    if _LINEAR_ACC is not torch.float32:
        return rbf((x.to(_LINEAR_ACC) @ w.t().to(_LINEAR_ACC)).float())
    return rbf(x @ w.t())


def rms_norm_qwen3(x, w, eps):
    """HF Qwen3RMSNorm: weight * bf16(x * rsqrt(mean(x^2) + eps)), bf16 product."""
    var = x.pow(2).mean(-1, keepdim=True)
    return rbf(w * rbf(x * torch.rsqrt(var + eps)))


def rms_norm_qwen35(x, w, eps):
    """HF Qwen3_5RMSNorm: bf16((x * rsqrt(mean(x^2) + eps)) * (1 + weight)) in fp32."""
    var = x.pow(2).mean(-1, keepdim=True)
    return rbf(x * torch.rsqrt(var + eps) * (1.0 + w))


def gated_rms_norm(x, z, w, eps):
    """HF Qwen3_5RMSNormGated as called in compiler/qwen35/adapters/delta.py:46-47:
    bf16( bf16(weight * bf16(x * rsqrt(mean(x^2) + eps))) * silu(z) )."""
    var = x.pow(2).mean(-1, keepdim=True)
    n = rbf(w * rbf(x * torch.rsqrt(var + eps)))
    return rbf(n * F.silu(z))


def silu_bf16(x):
    """F.silu on a bf16 tensor: fp32 math, bf16 result."""
    return rbf(F.silu(x))


def inv_freq(theta, rotary_dim):
    """HF default RoPE init: 1 / theta^(arange(0, dim, 2) / dim), fp32."""
    return 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).float() / rotary_dim))


def rope_tables(positions, inv):
    """cos/sin as bf16 values (compiler/qwen35/model.py:144-151; HF Qwen3 rotary module)."""
    freqs = positions.float()[:, None] * inv[None, :]
    cos, sin = rbf(freqs.cos()), rbf(freqs.sin())
    return torch.cat((cos, cos), -1), torch.cat((sin, sin), -1)


def apply_rope(x, cos, sin):
    """HF apply_rotary_pos_emb on bf16 tensors: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)),
    first cos.shape[-1] dims rotated, the rest passed through. x [..., D], cos/sin [..., RD]."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    half = rd // 2
    rot = torch.cat((-xr[..., half:], xr[..., :half]), -1)
    out = rbf(rbf(xr * cos) + rbf(rot * sin))
    return torch.cat((out, xp), -1)


def prefix_attention(q, k_cache, v_cache, length, scale):
    """Decode-row attention over cache[0:length] (attention.cpp:14-79; lower-right causal with
    T == 1 means the whole populated prefix). q [Hq, D], caches [Hkv, C, D]; GQA without expansion.

    Rounding points of the FlashAttention-2 kernel that attention.cpp:14-79 calls: fp32 scores
    and exponentials, the row sum taken over the fp32 probabilities, the probabilities rounded to
    bf16 for the P.V product (fp32 accumulation), the normalised output rounded to bf16."""
    hq, d = q.shape
    hkv = k_cache.shape[0]
    group = hq // hkv
    k = k_cache[:, :length].float()
    v = v_cache[:, :length].float()
    qg = q.view(hkv, group, d)
    scores = torch.einsum("hgd,hld->hgl", qg, k) * scale
    p = torch.exp(scores - scores.amax(-1, keepdim=True))
    lsum = p.sum(-1, keepdim=True)
    o = torch.einsum("hgl,hld->hgd", rbf(p), v) / lsum
    return rbf(o.reshape(hq, d))


def deltanet_core(qkv, b, a, conv, state, conv_w, a_log, dt_bias, active, hk, hv, dk):
    """One token of the Triton fused recurrence (recurrent.py:20-124) for one row.

    qkv [CH] bf16 values, b/a [HV], conv [CH, 4] bf16, state [HV, DK, DK] fp32 (rows = key dim,
    columns = value dim), conv_w [CH, 4]. Returns (core [HV*DK] bf16 values, next conv, next state).
    Empty rows (active False) keep both states and output zeros (recurrent.py:43-52,122).
    """
    if not active:
        return torch.zeros(hv * dk), conv.clone(), state.clone()
    window = torch.cat((conv[:, 1:], qkv[:, None]), dim=1)  # [CH, 4]: conv[1..3], x
    total = torch.zeros(window.shape[0])
    for tap in range(window.shape[1]):
        total = fma32(window[:, tap], conv_w[:, tap], total)
    v = rbf(total)
    mixed = rbf(v * (1.0 / (1.0 + torch.exp(-v))))  # SiLU as value * sigmoid(value), bf16
    next_conv = window.clone()
    q = mixed[: hk * dk].view(hk, dk)
    k = mixed[hk * dk : 2 * hk * dk].view(hk, dk)
    vv = mixed[2 * hk * dk :].view(hv, dk)
    scale = float(dk) ** -0.5
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * scale
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    beta = rbf(1.0 / (1.0 + torch.exp(-b)))
    x = a + dt_bias
    softplus = torch.where(x > 20.0, x, torch.log1p(torch.exp(x)))
    g = -torch.exp(a_log) * softplus
    group = hv // hk
    out = torch.zeros(hv, dk)
    new_state = torch.empty_like(state)
    for h in range(hv):
        kh = h // group
        s = state[h] * torch.exp(g[h])
        pred = (s * k[kh][:, None]).sum(0)
        delta = (vv[h] - pred) * beta[h]
        s = s + k[kh][:, None] * delta[None, :]
        out[h] = (s * q[kh][:, None]).sum(0)
        new_state[h] = s
    return rbf(out).view(-1), next_conv, new_state


def decode_step(geometry, W, input_ids, cache_position, state, kv_lengths, query_lengths):
    """ModelStep.forward at T == 1 for B rows.

    W: fp32 weights (prepare_weights). input_ids / cache_position: int64 [B]; kv_lengths /
    query_lengths: int [B]. state: list in the reference's order (per layer: key, value or
    conv, recurrent), rows [0, B). KV tensors are updated in place; conv / recurrent are returned
    as new tensors. Returns (logits bf16 [B, V], new_state list).
    """
    g = geometry
    q35 = g.family == "qwen3.5"
    norm = rms_norm_qwen35 if q35 else rms_norm_qwen3
    eps = g.rms_eps
    B = len(input_ids)
    inv = inv_freq(g.rope_theta, g.rotary_dim)
    new_state = list(state)
    hidden = W["model.embed_tokens.weight"][torch.as_tensor(input_ids)]  # [B, H]
    cos, sin = rope_tables(torch.as_tensor(cache_position), inv)
    active = [int(q) > 0 for q in query_lengths]
    for i in range(g.num_layers):
        p = f"model.layers.{i}."
        resid = hidden
        x = norm(hidden, W[p + "input_layernorm.weight"], eps)
        if g.is_delta(i):
            a_ = p + "linear_attn."
            qkv = linear(x, W[a_ + "in_proj_qkv.weight"])
            z = linear(x, W[a_ + "in_proj_z.weight"])
            bb = linear(x, W[a_ + "in_proj_b.weight"])
            aa = linear(x, W[a_ + "in_proj_a.weight"])
            conv_w = W[a_ + "conv1d.weight"].reshape(g.conv_channels, g.conv_width)
            conv_in, rec_in = state[2 * i], state[2 * i + 1]
            cores, convs, recs = [], [], []
            for r in range(B):
                c, nc, ns = deltanet_core(
                    qkv[r], bb[r], aa[r], conv_in[r].float(), rec_in[r].float(), conv_w,
                    W[a_ + "A_log"], W[a_ + "dt_bias"], active[r],
                    g.lin_key_heads, g.lin_value_heads, g.lin_head_dim,
                )
                cores.append(c)
                convs.append(nc)
                recs.append(ns)
            core = torch.stack(cores)
            new_state[2 * i] = torch.stack(convs).to(conv_in.dtype)
            new_state[2 * i + 1] = torch.stack(recs).to(rec_in.dtype)
            dv = g.lin_head_dim
            gn = gated_rms_norm(core.view(B, -1, dv), z.view(B, -1, dv), W[a_ + "norm.weight"], eps)
            out = linear(gn.view(B, -1), W[a_ + "out_proj.weight"])
        else:
            a_ = p + "self_attn."
            D, HQ, HKV = g.head_dim, g.num_q_heads, g.num_kv_heads
            qp = linear(x, W[a_ + "q_proj.weight"])
            if q35:
                qp = qp.view(B, HQ, 2 * D)
                query, gate = qp[..., :D], qp[..., D:].reshape(B, HQ * D)
            else:
                query, gate = qp.view(B, HQ, D), None
            key = linear(x, W[a_ + "k_proj.weight"]).view(B, HKV, D)
            value = linear(x, W[a_ + "v_proj.weight"]).view(B, HKV, D)
            query = norm(query, W[a_ + "q_norm.weight"], eps)
            key = norm(key, W[a_ + "k_norm.weight"], eps)
            query = apply_rope(query, cos[:, None, :], sin[:, None, :])
            key = apply_rope(key, cos[:, None, :], sin[:, None, :])
            kc, vc = state[2 * i], state[2 * i + 1]
            att = torch.zeros(B, HQ * D)
            for r in range(B):
                if not active[r]:
                    continue
                pos = int(cache_position[r])
                kc[r, :, pos] = key[r].to(kc.dtype)
                vc[r, :, pos] = value[r].to(vc.dtype)
                att[r] = prefix_attention(query[r], kc[r], vc[r], int(kv_lengths[r]),
                                          D ** -0.5).view(-1)
            if q35:
                att = rbf(att * rbf(torch.sigmoid(gate)))
            out = linear(att, W[a_ + "o_proj.weight"])
        hidden = rbf(resid + out)
        resid = hidden
        x = norm(hidden, W[p + "post_attention_layernorm.weight"], eps)
        gate_ = linear(x, W[p + "mlp.gate_proj.weight"])
        up = linear(x, W[p + "mlp.up_proj.weight"])
        act = rbf(silu_bf16(gate_) * up)
        hidden = rbf(resid + linear(act, W[p + "mlp.down_proj.weight"]))
    hidden = norm(hidden, W["model.norm.weight"], eps)
    logits = linear(hidden, W.get("lm_head.weight", W["model.embed_tokens.weight"]))
    logits[~torch.as_tensor(active)] = 0.0
    return logits.to(BF16), new_state


def argmax_first(logits):
    """torch.argmax on a bf16 row: first maximal index (generation.h:39)."""
    return torch.argmax(logits.float(), dim=-1)


def allocate_state(geometry, capacity, rows=8, fill=0.0):
    g = geometry
    out = []
    for i in range(g.num_layers):
        if g.is_delta(i):
            out.append(torch.zeros(rows, g.conv_channels, g.conv_width, dtype=BF16))
            out.append(torch.zeros(rows, g.lin_value_heads, g.lin_head_dim, g.lin_head_dim))
        else:
            kv = (rows, g.num_kv_heads, capacity, g.head_dim)
            out.append(torch.full(kv, fill, dtype=BF16))
            out.append(torch.full(kv, fill, dtype=BF16))
    return out


def run_tokens(geometry, W, tokens, capacity, state=None, start=0):
    """Teacher-forced single-row decode of `tokens` from position `start`; returns per-step
    logits and the final state."""
    state = state if state is not None else allocate_state(geometry, capacity, rows=1)
    logits = []
    for t, tok in enumerate(tokens):
        pos = start + t
        out, state = decode_step(geometry, W, [tok], [pos], state, [pos + 1], [1])
        logits.append(out[0])
    return torch.stack(logits), state


def cosine(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def rel_l2(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float((a - b).norm() / (b.norm() + 1e-30))


__all__ = [name for name in dir() if not name.startswith("_")]
_ = math
