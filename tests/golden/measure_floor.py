"""Measure the noise floor of the headline workload on the CPU oracle.

    python tests/golden/measure_floor.py [--out tests/golden/noise_floor.json]

Workload (the bench's headline): full-depth Qwen3.5-0.8B, seeded random-init bf16 weights
(xinfer_b200/synthetic.py, seed 0, no norm jitter), KV capacity 4096, a 512-token uniform random
prompt fed one token per step, then 8 more teacher-forced decode steps. The oracle runs twice:
once with fp32 sums in every linear (the reference's accumulation type) and once with fp64 sums.
Both are valid roundings of the same model; their difference is how far two legitimate
summation orders drift apart over this workload. The script records, per step, the logits'
max-abs difference and cosine, the greedy-token agreement, and at the end the state's relative
L2 difference and the KV slots' agreement (bitwise fraction, ulp distances). It does the same
for the schedules of the full-size reference fixtures in this folder. tests/test_headline_gpu.py
and tests/test_decode_gpu.py hold the CUDA kernel to twice these figures. Takes about 15
minutes on 8 cores.
"""

import argparse
import json
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle import qwen_step as O  # noqa: E402
from xinfer_b200 import configs, synthetic  # noqa: E402

CONFIG, CAPACITY, PROMPT, DECODE = "qwen3.5-0.8b", 4096, 512, 8
PROMPT_SEED, DECODE_SEED = 2024, 2025


def workload_tokens(g):
    """The teacher-forced token ids: the prompt, then DECODE further random ids."""
    return (synthetic.random_prompt(g, PROMPT, seed=PROMPT_SEED)
            + synthetic.random_prompt(g, DECODE, seed=DECODE_SEED))


def bf16_ulps(a, b):
    """Distance in bf16 units in the last place between two bf16 tensors (ordered bit patterns)."""
    def ordered(t):
        i = t.contiguous().view(torch.int16).int()
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (ordered(a) - ordered(b)).abs()


def compare(g, a, sa, b, sb, n):
    """Per-step logits figures and end-of-run state figures of two runs over n positions."""
    steps = []
    for s in range(a.shape[0]):
        x, y = a[s].float(), b[s].float()
        ax, ay = int(O.argmax_first(a[s])), int(O.argmax_first(b[s]))
        steps.append({"max_abs": (x - y).abs().max().item(), "cosine": O.cosine(x, y),
                      "argmax_equal": ax == ay})
    rec, conv, ulps, kv_a, kv_b = [], [], [], [], []
    for i in range(g.num_layers):
        if g.is_delta(i):
            conv.append(O.rel_l2(sa[2 * i], sb[2 * i]))
            rec.append(O.rel_l2(sa[2 * i + 1], sb[2 * i + 1]))
        else:
            for j in (2 * i, 2 * i + 1):
                u, v = sa[j][:, :, :n], sb[j][:, :, :n]
                ulps.append(bf16_ulps(u, v).flatten())
                kv_a.append(u.float().flatten())
                kv_b.append(v.float().flatten())
    out = {
        "max_abs_all": max(s["max_abs"] for s in steps),
        "min_cosine_all": min(s["cosine"] for s in steps),
        "argmax_disagreements": sum(not s["argmax_equal"] for s in steps),
        "recurrent_rel_l2_max": max(rec) if rec else 0.0,
        "conv_rel_l2_max": max(conv) if conv else 0.0,
        "per_step": steps,
    }
    if ulps:
        u = torch.cat(ulps)
        out.update({"kv_bitwise_fraction": float((u == 0).float().mean()),
                    "kv_within_1ulp": float((u <= 1).float().mean()),
                    "kv_within_2ulp": float((u <= 2).float().mean()),
                    "kv_max_ulp": int(u.max()),
                    "kv_rel_l2": O.rel_l2(torch.cat(kv_a), torch.cat(kv_b))})
    return out


def run_schedule(g, W, schedule, capacity, dtype):
    rows = len(schedule[0])
    state = O.allocate_state(g, capacity, rows=rows)
    positions = [0] * rows
    out = []
    with O.accumulate(dtype):
        for tokens in schedule:
            ids = [t[0] if t else 0 for t in tokens]
            kv = [positions[r] + len(tokens[r]) for r in range(rows)]
            logits, state = O.decode_step(g, W, ids, positions[:], state, kv, [len(t) for t in tokens])
            out.append(logits[0].clone())
            for r in range(rows):
                positions[r] += len(tokens[r])
    return torch.stack(out), state


def run(g, W, tokens, dtype):
    state = O.allocate_state(g, CAPACITY, rows=1)
    out = []
    with O.accumulate(dtype):
        for pos, tok in enumerate(tokens):
            logits, state = O.decode_step(g, W, [tok], [pos], state, [pos + 1], [1])
            out.append(logits[0].clone())
    return torch.stack(out), state


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent / "noise_floor.json"))
    ap.add_argument("--skip-headline", action="store_true")
    args = ap.parse_args()
    torch.set_num_threads(8)
    result = {}
    t0 = time.time()
    if not args.skip_headline:
        g = configs.get(CONFIG)
        W = O.prepare_weights(synthetic.make_state_dict(g, seed=0))
        tokens = workload_tokens(g)
        a, sa = run(g, W, tokens, torch.float32)
        b, sb = run(g, W, tokens, torch.float64)
        head = compare(g, a, sa, b, sb, len(tokens))
        dec = head["per_step"][PROMPT:]
        head.update({"config": CONFIG, "capacity": CAPACITY, "prompt": PROMPT, "decode": DECODE,
                     "prompt_seed": PROMPT_SEED, "decode_seed": DECODE_SEED,
                     "max_abs_decode": max(s["max_abs"] for s in dec),
                     "min_cosine_decode": min(s["cosine"] for s in dec)})
        result["headline"] = head
        del W
    fixtures = {}
    here = Path(__file__).resolve().parent
    for name in ("qwen3-0.6b-short", "qwen3.5-0.8b-short", "qwen3.5-0.8b-cap4096"):
        fx = torch.load(here / f"{name}.pt", weights_only=False)
        g = configs.get(fx["config"])
        W = O.prepare_weights(synthetic.make_state_dict(g, seed=fx["seed"], jitter=fx["jitter"]))
        a, sa = run_schedule(g, W, fx["schedule"], fx["capacity"], torch.float32)
        b, sb = run_schedule(g, W, fx["schedule"], fx["capacity"], torch.float64)
        fixtures[name] = compare(g, a, sa, b, sb, len(fx["schedule"]))
        del W
    result["fixtures"] = fixtures
    result["seconds"] = time.time() - t0
    Path(args.out).write_text(json.dumps(result, indent=1) + "\n")
    brief = {k: {kk: vv for kk, vv in v.items() if kk != "per_step"} for k, v in fixtures.items()}
    if "headline" in result:
        brief["headline"] = {k: v for k, v in result["headline"].items() if k != "per_step"}
    print(json.dumps(brief, indent=1))


if __name__ == "__main__":
    main()
