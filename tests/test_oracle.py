"""Pin the CPU oracle: against fixtures produced by running the reference's own decode step
(tests/golden/make_golden.py) and against the known-answer cases of the reference's tests."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qwen_step as O
from xinfer_b200 import configs, synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(p.stem for p in GOLDEN.glob("*.pt"))
LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999
STATE_REL = 1e-2


def run_oracle(fx, dtype=torch.float32):
    """The oracle over a fixture's schedule; a step whose single row carries several tokens (a
    prefill chunk) is fed one token at a time, and its logits are the last token's."""
    g = configs.get(fx["config"])
    sd = synthetic.make_state_dict(g, seed=fx["seed"], jitter=fx["jitter"])
    W = O.prepare_weights(sd)
    rows = len(fx["schedule"][0])
    state = O.allocate_state(g, fx["capacity"], rows=rows)
    positions = [0] * rows
    logits = []
    with O.accumulate(dtype):
        for tokens in fx["schedule"]:
            width = max(len(t) for t in tokens)
            assert width <= 1 or rows == 1, "prefill chunks are single-row"
            for j in range(max(1, width)):
                ids = [t[j] if len(t) > j else 0 for t in tokens]
                kv = [positions[r] + min(len(tokens[r]), j + 1) for r in range(rows)]
                q = [1 if len(t) > j else 0 for t in tokens]
                out, state = O.decode_step(g, W, ids, [positions[r] + j for r in range(rows)], state, kv, q)
            logits.append(out)
            for r in range(rows):
                positions[r] += len(tokens[r])
    return g, torch.stack(logits), state, positions


@pytest.mark.parametrize("name", [f for f in FIXTURES if "0.6b" not in f and "0.8b" not in f
                                  and "prefill" not in f])
def test_oracle_matches_reference_fixture(name):
    fx = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    g, logits, state, positions = run_oracle(fx)
    assert positions == fx["positions"]
    ref = fx["logits"]
    for s, tokens in enumerate(fx["schedule"]):
        for r, t in enumerate(tokens):
            if not t:
                assert torch.count_nonzero(logits[s, r]) == 0 and torch.count_nonzero(ref[s, r]) == 0
                continue
            a, b = logits[s, r].float(), ref[s, r].float()
            err = ((a - b).abs() - (LOGIT_MAX_ABS + b.abs() * 2.0 ** -7)).max().item()
            cos = O.cosine(a, b)
            assert err <= 0 and cos >= LOGIT_COS, (s, r, err, cos)
            # greedy token: equal, or a near-tie in the reference's own logits (the reference's
            # validation also treats top-1 flips inside the numeric margin as diagnostics)
            mine, theirs = int(O.argmax_first(logits[s, r])), int(O.argmax_first(ref[s, r]))
            margin = float(ref[s, r, theirs].float() - ref[s, r, mine].float())
            assert mine == theirs or margin <= LOGIT_MAX_ABS, (s, r, mine, theirs, margin)
    # first step from zero state: every rounding point agrees, so logits are bit-equal up to a
    # rare one-ulp flip of an fp32 reduction (which then spreads one ulp through later layers)
    first = fx["schedule"][0]
    for r0 in (r for r, t in enumerate(first) if t):
        err0 = (logits[0, r0].float() - ref[0, r0].float()).abs().max().item()
        assert err0 <= 1e-2 and O.cosine(logits[0, r0], ref[0, r0]) >= 0.99995, (r0, err0)
    for i, smp in enumerate(fx["state_sample"]):
        got = state[i].reshape(-1)[smp["index"].long()]
        assert O.rel_l2(got.float(), smp["value"].float()) <= STATE_REL, i
    if fx["conv_state"] is not None and fx["conv_state"]:
        first_conv = next(i for i in range(g.num_layers) if g.is_delta(i))
        got = state[2 * first_conv]
        frac = (got == fx["conv_state"][0]).float().mean().item()
        assert frac >= 0.999, f"layer-0 conv state bitwise fraction {frac}"


# Full-depth random-init models amplify a single one-ulp bf16 flip of any fp32 sum: two valid
# accumulation orders of this very oracle (fp32 against fp64 sums in every linear) drift apart
# step by step by the figures of tests/golden/noise_floor.json (tests/golden/measure_floor.py).
# The oracle is held to twice that floor against the reference's full-depth fixtures, step by
# step; the north-star bar (2e-2, 0.9999) applies wherever the floor is below it.
FLOOR = json.loads((GOLDEN / "noise_floor.json").read_text())


def floor_bounds(per_step, window=16):
    """(max-abs, cosine) bound per step: twice the largest twin difference within `window` steps
    of it (one step's difference is a single sample of the spread), never tighter than the
    north-star bar needs."""
    out = []
    for s in range(len(per_step)):
        near = per_step[max(0, s - window):s + window + 1]
        mx = max(st["max_abs"] for st in near)
        mc = max(1.0 - st["cosine"] for st in near)
        out.append((max(LOGIT_MAX_ABS, 2.0 * mx), min(LOGIT_COS, 1.0 - 2.0 * mc)))
    return out


@pytest.mark.parametrize("name", [f for f in FIXTURES if "0.6b" in f or "0.8b" in f])
def test_oracle_matches_full_size_fixture(name):
    fx = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    g, logits, state, _ = run_oracle(fx)
    floor = FLOOR["fixtures"][name]
    bounds = floor_bounds(floor["per_step"])
    summ = fx["logits_summary"]
    tail = fx.get("logits_tail")
    tail0 = len(fx["schedule"]) - (tail.shape[0] if tail is not None else 0)
    for s in range(len(fx["schedule"])):
        bmax, bcos = bounds[s]
        idx = summ["top_indices"][s, 0]
        err = (logits[s, 0].float()[idx] - summ["top_values"][s, 0].float()).abs().max().item()
        assert err <= bmax, (s, err, bmax)
        sl = logits[s, 0, ::97].float()
        assert O.cosine(sl, summ["stride_slice"][s, 0]) >= bcos
        assert (sl - summ["stride_slice"][s, 0].float()).abs().max().item() <= bmax
        if tail is not None and s >= tail0:
            a, b = logits[s, 0].float(), tail[s - tail0, 0].float()
            assert (a - b).abs().max().item() <= bmax and O.cosine(a, b) >= bcos, s
            mine, theirs = int(a.argmax()), int(b.argmax())
            assert mine == theirs or float(b[theirs] - b[mine]) <= bmax, (s, mine, theirs)
    rel = max(STATE_REL, 2 * floor["recurrent_rel_l2_max"], 2 * floor["conv_rel_l2_max"],
              2 * floor.get("kv_rel_l2", 0.0))
    for i, smp in enumerate(fx["state_sample"]):
        got = state[i].reshape(-1)[smp["index"].long()]
        assert O.rel_l2(got.float(), smp["value"].float()) <= rel, i


def test_noise_floor_record_matches_its_workload():
    """The floor record names the workload the headline GPU test runs."""
    head = FLOOR["headline"]
    assert (head["config"], head["capacity"], head["prompt"], head["decode"]) == ("qwen3.5-0.8b", 4096, 512, 8)
    assert len(head["per_step"]) == head["prompt"] + head["decode"]
    assert set(FLOOR["fixtures"]) >= {f for f in FIXTURES if "0.6b" in f or "0.8b" in f}


@pytest.mark.parametrize("name", [f for f in FIXTURES if "prefill" in f])
def test_oracle_matches_reference_prefill_fixture(name):
    """The reference's own 128-token prefill chunk (its chunk-64 DeltaNet path, recurrent.py:234-281,
    chunked.py) against the oracle's token-by-token recurrence: the same gated delta rule summed in
    another order. Held to the north-star bar, or twice the spread of the oracle against its own
    fp64-sum twin on this schedule where that is larger."""
    fx = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    g, logits, state, positions = run_oracle(fx)
    _, twin, tstate, _ = run_oracle(fx, torch.float64)
    assert positions == fx["positions"]
    for s in range(len(fx["schedule"])):
        a, b, c = logits[s, 0].float(), fx["logits"][s, 0].float(), twin[s, 0].float()
        spread = (a - c).abs().max().item()
        bound = max(LOGIT_MAX_ABS, 2 * spread)
        assert ((a - b).abs() - (bound + b.abs() * 2.0 ** -7)).max().item() <= 0, (s, (a - b).abs().max().item())
        assert O.cosine(a, b) >= min(LOGIT_COS, 1 - 2 * (1 - O.cosine(a, c))), s
    for i, smp in enumerate(fx["state_sample"]):
        got = state[i].reshape(-1)[smp["index"].long()]
        tw = tstate[i].reshape(-1)[smp["index"].long()]
        assert O.rel_l2(got.float(), smp["value"].float()) <= max(STATE_REL, 2 * O.rel_l2(tw.float(), got.float()) + 1e-3), i


def test_attention_lower_right_causality_kat():
    """compiler/common/tests/test_attention.py:293-307: q = k = 0, v[pos] = pos, extent 5 ->
    the last query (decode row) averages positions 0..4 = 2.0; with two appended queries the
    earlier one sees 0..3 (1.5). The decode oracle covers the T == 1 row."""
    for hq, hkv, d in ((16, 8, 128), (8, 2, 256)):
        q = torch.zeros(hq, d)
        k = torch.zeros(hkv, 16, d, dtype=torch.bfloat16)
        v = torch.arange(16, dtype=torch.bfloat16)[None, :, None].expand(hkv, 16, d).contiguous()
        out = O.prefix_attention(q, k, v, 5, d ** -0.5)
        assert torch.equal(out, torch.full((hq, d), 2.0))
        out = O.prefix_attention(q, k, v, 4, d ** -0.5)
        assert torch.equal(out, torch.full((hq, d), 1.5))


def _fma32(a, b, c):
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def _bf16(x):
    return float(torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).float())


def test_deltanet_conv_cancellation_kat():
    """compiler/qwen35/tests/delta.py:185-191: exact bf16 conv constants whose products cancel;
    the conv sum must be rounded to bf16 before SiLU and the SiLU result rounded again."""
    conv = [0.99609375, -1.0078125, 0.50390625, -0.49609375]
    weight = [0.333984375, 0.333984375, -0.66796875, -0.66796875]
    x = 0.498046875
    window = conv[1:] + [x]
    total = np.float32(0.0)
    for h, w in zip(window, weight):
        total = _fma32(h, w, total)
    v = _bf16(float(total))
    expect = _bf16(float(np.float32(v) * (np.float32(1.0) / (np.float32(1.0) + np.exp(np.float32(-v))))))
    hk, hv, dk = 16, 16, 128
    ch = (2 * hk + hv) * dk
    c, next_conv, _ = O.deltanet_core(
        torch.full((ch,), x), torch.zeros(hv), torch.zeros(hv),
        torch.tensor(conv).repeat(ch, 1), torch.zeros(hv, dk, dk), torch.tensor(weight).repeat(ch, 1),
        torch.full((hv,), -2.0), torch.zeros(hv), True, hk, hv, dk)
    assert torch.equal(next_conv[0], torch.tensor(window))
    # value channels go straight to the delta rule: with zero state, out = (k.q) * beta * v
    # so check the rounded conv value through an identity path: recompute mixed directly
    window_t = torch.tensor(window)[None].repeat(ch, 1)
    tot = torch.zeros(ch)
    for tap in range(4):
        tot = O.fma32(window_t[:, tap], torch.tensor(weight)[tap].expand(ch), tot)
    vv = O.rbf(tot)
    mixed = O.rbf(vv * (1.0 / (1.0 + torch.exp(-vv))))
    assert float(mixed[0]) == expect


def test_deltanet_gate_extremes_match_float64():
    """compiler/qwen35/tests/delta.py:161-179: b = linspace(-80, 80), a in {-80 .. 80}."""
    hk, hv, dk = 16, 16, 128
    ch = (2 * hk + hv) * dk
    gen = torch.Generator().manual_seed(0)
    for a_val in (-80.0, -20.0, -1.0, 0.0, 19.0, 20.0, 21.0, 80.0):
        qkv = torch.randn(ch, generator=gen).to(torch.bfloat16).float()
        conv = (torch.randn(ch, 4, generator=gen) * 0.3).to(torch.bfloat16).float()
        wc = (torch.randn(ch, 4, generator=gen) * 0.2).to(torch.bfloat16).float()
        state = torch.randn(hv, dk, dk, generator=gen) * 0.1
        b = torch.linspace(-80, 80, hv).to(torch.bfloat16).float()
        a = torch.full((hv,), a_val)
        a_log = torch.full((hv,), -2.0)
        dt = (torch.randn(hv, generator=gen) * 0.1).to(torch.bfloat16).float()
        core, _, final = O.deltanet_core(qkv, b, a, conv, state, wc, a_log, dt, True, hk, hv, dk)
        assert torch.isfinite(core).all() and torch.isfinite(final).all()
        x = (a + dt).double()
        sp = torch.where(x > 20, x, torch.log1p(torch.exp(x)))
        decay = torch.exp(-torch.exp(a_log.double()) * sp)
        assert (decay >= 0).all()


def test_rope_tables_match_hf_rotary():
    """Text RoPE: compiler/qwen35/model.py:144-151 (bitwise vs HF in the reference's tests)."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding

    g = configs.QWEN35_0_8B
    hf = configs.hf_config(g)
    rot = Qwen3_5TextRotaryEmbedding(hf)
    pos = torch.tensor([0, 1, 7, 511, 4095, 16383])
    cos, sin = O.rope_tables(pos, O.inv_freq(g.rope_theta, g.rotary_dim))
    hc, hs = rot(torch.zeros(1, dtype=torch.bfloat16), pos[None])
    assert torch.equal(cos.to(torch.bfloat16), hc[0]) and torch.equal(sin.to(torch.bfloat16), hs[0])
    assert torch.equal(O.inv_freq(g.rope_theta, g.rotary_dim), rot.inv_freq)


def test_argmax_first_index_and_nan():
    row = torch.tensor([1.0, 3.0, 3.0, 2.0], dtype=torch.bfloat16)
    assert int(O.argmax_first(row)) == 1
    row = torch.tensor([1.0, float("nan"), 3.0, float("nan")], dtype=torch.bfloat16)
    assert int(O.argmax_first(row)) == 1


# SHA-256 of the bf16 bytes of synthetic tensors (qwen3.5-tiny, seed 0, jitter 0.1) as this
# recipe produced them when the committed fixtures were made: pins the generator across machines
# and torch versions (a change here invalidates every fixture under tests/golden).
SYNTHETIC_SHA256 = {
    "model.embed_tokens.weight": "33eff2605f2c0b73f020f5ec6db112ebfe6b2fbf934c8c8f04a8b671875f801d",
    "model.layers.0.linear_attn.in_proj_qkv.weight":
        "988739fe60162b77dcc3806af51246a4ee572502cc720b7b8710c45ac711bb9d",
    "model.layers.0.linear_attn.A_log": "656705c79a95826cdcc3d44a997c3f43c9d32cf91826cf10fa59b151e6b9159c",
    "model.layers.3.self_attn.q_norm.weight":
        "00a35034db129a8346a337a7b884494d96d619a0a11f38e7cc7f15a39b8e75b0",
}


def test_synthetic_recipe_is_stable():
    g = configs.QWEN35_TINY
    a = synthetic.make_state_dict(g, seed=0, jitter=0.1)
    for name, digest in SYNTHETIC_SHA256.items():
        got = hashlib.sha256(a[name].view(torch.int16).numpy().tobytes()).hexdigest()
        assert got == digest, name
    w = a["model.layers.0.linear_attn.in_proj_qkv.weight"].float()
    assert abs(w.std().item() - 0.02) < 1e-3
