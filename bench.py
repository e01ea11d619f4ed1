"""Decode throughput of the B200 megakernel on BASELINE's headline workload.

Workload (the metric's config): Qwen3.5-0.8B hybrid text model, seeded
random-init bf16 weights, batch 1, a 512-token uniform-random prompt, then greedy decode at
4096-slot KV capacity with carried conv / recurrent state. One bench "step" = one decode token
(one launch of the persistent decode kernel).

  value  device-timed tokens/s of the K timed steps, inputs resident in HBM (each step's token
         is the previous step's fused argmax, read on the device)
  e2e    the same metric through the public runner path with host buffers: per step a pinned
         host->device copy of token id + position and a device->host read of the next token,
         then a host sync (wall clock over the K steps)
  roofline  algorithmic bytes per token / mean launch time vs the measured HBM copy peak
  cpu_baseline  the unchanged HF transformers model, eager, bf16, on this host's cores, with the
         call pattern of the reference's HF benchmark worker (tools/benchmark/common.py:237-267):
         the whole prompt in one call (untimed), then one forced token per call with
         logits_to_keep=1, argmax and host read per step; all host threads, and the 1-thread
         figure (the reference's thread policy) beside it. The fp32 CPU oracle's decode rate is
         reported as a secondary figure.
Multi-GPU (torchrun, one process per GPU): independent replicas, no collective on the data
path; the timed region is bracketed by barriers and the slowest rank's time is reported.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "decode tok/s at batch 1 (Qwen3.5-0.8B, 4K ctx); % of HBM roofline"
UNIT = "tokens/s"
PROFILE = ROOT / "profiles" / "decode_megakernel_qwen3.5-0.8b.md"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="qwen3.5-0.8b")
    ap.add_argument("--prompt", type=int, default=512,
                    help="prompt length (batch > 1: the largest of the rows' random lengths)")
    ap.add_argument("--batch", type=int, default=1, help="rows per GPU, 1..8, ragged prompts")
    ap.add_argument("--capacity", type=int, default=4096)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="budget of the secondary CPU-oracle figure")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--trace", help="save a per-CTA stage trace of one extra step to this file")
    ap.add_argument("--measure", choices=("decode", "prefill"), default="decode",
                    help="prefill: time the prompt's 512-token prefill chunks instead (tokens/s and "
                         "tensor-pipe utilisation of the projections)")
    return ap.parse_args()


def max_over_ranks(x, dist, device):
    """The slowest replica's figure: a job of independent replicas ends with its slowest rank."""
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(world, steps, seconds):
    """Tokens per second of the whole job: each of `world` replicas decodes `steps` tokens."""
    return world * steps / seconds


def workload(args):
    rows = (f"batch 1, {args.prompt}-token random prompt" if args.batch == 1 else
            f"batch {args.batch} ragged rows, prompts U[2,{args.prompt}]")
    return f"{args.config} decode, {rows} per GPU, {args.capacity}-slot capacity"


def algorithmic_bytes(g, contexts):
    """Bytes one decode step must move: every weight once (tied lm_head counted once, embedding
    rows excluded), then per active row its recurrent + conv state read and written, its KV prefix
    read plus one slot written. `contexts`: cached positions per row (a number for one row)."""
    from xinfer_b200 import synthetic

    if not isinstance(contexts, (list, tuple)):
        contexts = [contexts]
    total = 0
    for name, (shape, _) in synthetic.parameter_shapes(g).items():
        if name == "model.embed_tokens.weight":
            continue
        n = 1
        for s in shape:
            n *= s
        total += 2 * n
    total += 2 * g.vocab * g.hidden  # lm_head (tied to the embedding)
    n_delta = sum(g.is_delta(i) for i in range(g.num_layers))
    n_attn = g.num_layers - n_delta
    rec = g.lin_value_heads * g.lin_head_dim * g.lin_head_dim * 4
    conv = g.conv_channels * g.conv_width * 2
    kv_token = 2 * g.num_kv_heads * g.head_dim * 2
    for context in contexts:
        total += n_delta * 2 * (rec + conv)
        total += n_attn * kv_token * (context + 1)
    return total


def prefill_flops(g, chunks):
    """Algorithmic FLOPs of prefilling chunks [(start, T), ...]: every projection of every layer
    (2 K N per token; the packed in_proj, q|k|v, o/out_proj, gate, up, down), the prefix attention
    (4 D per visible key and query head: Q.K^T and P.V) and the DeltaNet scan (about 8 dk dv per
    token and value head), and the lm_head of the last token only."""
    H, I = g.hidden, g.intermediate
    per_token = 0
    attn = 0
    for i in range(g.num_layers):
        if g.is_delta(i):
            hv = g.lin_value_heads * g.lin_head_dim
            per_token += 2 * H * (g.conv_channels + hv + 2 * g.lin_value_heads) + 2 * hv * H
            per_token += 8 * g.lin_value_heads * g.lin_head_dim * g.lin_head_dim
        else:
            per_token += 2 * H * (g.q_rows + 2 * g.num_kv_heads * g.head_dim) + 2 * g.num_q_heads * g.head_dim * H
            attn += 1
        per_token += 2 * H * 2 * I + 2 * I * H
    total = 0
    for start, T in chunks:
        total += per_token * T
        # keys visible to query t: start + t + 1
        total += attn * 4 * g.head_dim * g.num_q_heads * (T * start + T * (T + 1) // 2)
    return total + 2 * g.vocab * H


def measure_prefill(args, dist, dev, world, rank):
    """Prefill throughput of the prompt in 512-token chunks."""
    from xinfer_b200 import configs, synthetic
    from xinfer_b200.engine import Engine, pack_linears

    g = configs.get(args.config)
    # the reference bundle's layout: each projection group as adjacent rows of one tensor
    weights = pack_linears(g, synthetic.make_state_dict(g, seed=0, device=dev))
    eng = Engine(g, weights, capacity=args.capacity, device=dev)
    prompt = synthetic.random_prompt(g, args.prompt, seed=1000 + rank)
    ids = torch.tensor(prompt, dtype=torch.int64).to(dev)
    state = [t.narrow(0, 0, 1) for t in eng.allocate_state()]
    logits = torch.empty(g.vocab, dtype=torch.bfloat16, device=dev)
    nxt = torch.empty(1, dtype=torch.int64, device=dev)
    chunks = [(c, min(512, args.prompt - c)) for c in range(0, args.prompt, 512)]
    stream = torch.cuda.current_stream(dev)

    def run_prompt():
        for start, T in chunks:
            eng.prefill(ids[start:start + T], start, state, state, logits, nxt)

    for _ in range(max(1, args.warmup)):
        run_prompt()
    eng.check_prefill_error()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps)
    with Clocks(dev.index or 0) as clocks:
        ev0.record(stream)
        for _ in range(steps):
            run_prompt()
        ev1.record(stream)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
    ms = max_over_ranks(ev0.elapsed_time(ev1), dist, dev)
    eng.check_prefill_error()
    tokens = steps * args.prompt
    flops = steps * prefill_flops(g, chunks)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    achieved = flops / (ms / 1000.0) / 1e12
    line = {
        "metric": f"prefill tok/s ({args.config}, {args.prompt}-token prompt in 512-token chunks)",
        "value": job_throughput(world, tokens, ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.config} prefill of a {args.prompt}-token random prompt per GPU in "
                               f"{len(chunks)} chunks, {args.capacity}-slot capacity",
                   "model": args.config, "global_batch": world, "seq_len": args.capacity},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_kind": "measured" if peaks else "fallback",
                     "algorithmic_flops_per_step": flops / steps},
        "clocks": clocks.summary(),
    }
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profile(g, context):
    """DRAM bytes per launch from the committed ncu capture (dram__bytes_read.sum +
    dram__bytes_write.sum), moved from the captured KV length to this run's mean context by the
    KV bytes of the attention layers (the only traffic that depends on the context)."""
    if not PROFILE.exists() or g.name != "qwen3.5-0.8b":
        return None
    fields = {}
    for line in PROFILE.read_text().splitlines():
        key, _, rest = line.strip().partition(":")
        if key in ("traffic_bytes_per_launch", "traffic_kv_len") and rest.strip():
            try:
                fields[key] = float(rest.split()[0])
            except ValueError:
                return None
    if len(fields) != 2:
        return None
    n_attn = sum(not g.is_delta(i) for i in range(g.num_layers))
    kv_token = 2 * g.num_kv_heads * g.head_dim * 2
    return fields["traffic_bytes_per_launch"] + n_attn * kv_token * (context + 1 - fields["traffic_kv_len"])


class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        mhz, max_mhz, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        top = sorted(mhz)[len(mhz) // 4:] or mhz  # samples under load
        return {"sm_mhz": statistics.median(top), "sm_max_mhz": max_mhz, "reasons": sorted(reasons),
                "samples": len(mhz)}


def hf_eager_model(g):
    """The unchanged HF text model, built as the reference's loaders build it
    (compiler/qwen35/model.py:21-42, compiler/qwen3/model.py:16-26): sdpa attention, bf16, tied
    lm_head, RoPE buffers recreated in fp32; the seeded synthetic weights of the GPU run instead
    of a checkpoint; on the CPU."""
    from xinfer_b200 import configs, synthetic

    hf = configs.hf_config(g)
    hf._attn_implementation = "sdpa"
    cpu_kernels = {}
    if g.family == configs.QWEN35:
        from transformers import Qwen3_5ForCausalLM as Model
        from transformers.models.qwen3_5 import modeling_qwen3_5 as hf_module
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding as Rotary
        # the CPU build HF makes when the GPU-only fla / causal-conv1d kernels are absent: its
        # torch Gated DeltaNet (chunked prefill, recurrent decode, conv update) and gated norm
        cpu_kernels = {"FusedRMSNormGated": None, "chunk_gated_delta_rule": None,
                       "fused_recurrent_gated_delta_rule": None, "causal_conv1d_fn": None,
                       "causal_conv1d_update": None, "is_fast_path_available": False}
    else:
        from transformers import Qwen3ForCausalLM as Model
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding as Rotary
        hf_module = None
    saved = {name: getattr(hf_module, name) for name in cpu_kernels}
    try:
        for name, value in cpu_kernels.items():
            setattr(hf_module, name, value)
        with torch.device("meta"):
            model = Model(hf)
    finally:
        for name, value in saved.items():
            setattr(hf_module, name, value)
    model.load_state_dict(synthetic.make_state_dict(g, seed=0), strict=True, assign=True)
    model.lm_head.weight = model.model.embed_tokens.weight
    model.model.rotary_emb = Rotary(hf)
    return model.eval().requires_grad_(False)


def hf_eager_baseline(g, prompt_len, steps, warmup, threads_list):
    """Decode tokens/s of the HF eager model on the CPU, one figure per thread count.

    The reference's HF worker (tools/benchmark/common.py:237-267, measured as measure_request at
    :94-121): HF owns the cache; the whole prompt goes in one call; then one forced token per
    call with logits_to_keep=1, each followed by the argmax and its host read. The prompt is the
    GPU run's (seeded uniform random ids, same length) and is prefilled with all host threads as
    untimed set-up; the forced decode tokens are seeded random ids."""
    from xinfer_b200 import synthetic

    all_threads = len(os.sched_getaffinity(0))
    model = hf_eager_model(g)
    prompt = synthetic.random_prompt(g, prompt_len, seed=1000)
    forced = synthetic.random_prompt(g, (steps + warmup) * len(threads_list), seed=77)
    rates = {}
    with torch.inference_mode():
        torch.set_num_threads(all_threads)
        out = model(input_ids=torch.tensor([prompt]), past_key_values=None, use_cache=True,
                    logits_to_keep=1)
        cache = out.past_key_values
        out.logits[:, -1, :].argmax(-1).item()
        k = 0
        for threads in threads_list:
            torch.set_num_threads(threads)
            times = []
            for _ in range(warmup + steps):
                t0 = time.perf_counter()
                out = model(input_ids=torch.tensor([[forced[k]]]), past_key_values=cache,
                            use_cache=True, logits_to_keep=1)
                cache = out.past_key_values
                out.logits[:, -1, :].argmax(-1).item()
                times.append(time.perf_counter() - t0)
                k += 1
            rates[threads] = steps / sum(times[warmup:])
    torch.set_num_threads(all_threads)
    return rates, prompt_len + k


def cpu_baseline(args, g, steps=8, warmup=2):
    """The HF eager CPU baseline at the GPU run's context (all threads, then 1 thread)."""
    threads = len(os.sched_getaffinity(0))
    rates, end = hf_eager_baseline(g, max(1, args.prompt), steps, warmup, [threads, 1])
    return {"value": rates[threads], "unit": UNIT, "cores": threads, "kind": "reference",
            "value_1_thread": rates[1],
            "sample": f"HF transformers eager {args.config} (bf16, sdpa, HF cache) on the CPU with the "
                      f"call pattern of the reference's HF benchmark worker: a {args.prompt}-token "
                      f"prompt in one call (untimed), then {warmup} + {steps} forced decode tokens "
                      f"per thread count, one per call with logits_to_keep=1, argmax and host read "
                      f"per step, contexts {args.prompt + 1}..{end}; value: {threads} threads; "
                      f"value_1_thread: 1 thread (the reference's policy)"}


def oracle_port_rate(args, g, budget_s):
    """The CPU oracle (port of the reference step) on this host: decode tokens of the same model
    at a short context until the budget is spent (a secondary figure beside the HF baseline)."""
    from oracle import qwen_step as O
    from xinfer_b200 import synthetic

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    sd = synthetic.make_state_dict(g, seed=0)
    W = O.prepare_weights(sd)
    del sd
    state = O.allocate_state(g, 64, rows=1)
    prompt = synthetic.random_prompt(g, 64, seed=0)
    O.decode_step(g, W, [prompt[0]], [0], state, [1], [1])  # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < 63 and (time.perf_counter() - t0 < budget_s or n < 2):
        _, state = O.decode_step(g, W, [prompt[n + 1]], [n + 1], state, [n + 2], [1])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} decode tokens of the fp32 CPU oracle at context 2..{n + 1} on "
                      f"{threads} threads"}


def hf_eager_baseline_one_thread(g, args, steps):
    rates, end = hf_eager_baseline(g, max(1, args.prompt), steps, 1, [1])
    return rates[1], end


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from xinfer_b200 import configs

    g = configs.get(args.config)
    # all host threads for the timed steps, then a shorter 1-thread sample (the reference's policy)
    threads = len(os.sched_getaffinity(0))
    steps, warmup = max(1, args.steps), max(1, args.warmup)
    rates, end = hf_eager_baseline(g, max(1, args.prompt), steps, warmup, [threads])
    one, _ = hf_eager_baseline_one_thread(g, args, min(steps, 4))
    value = rates[threads]
    res = {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "value_1_thread": one,
           "sample": f"HF transformers eager {args.config} (bf16, sdpa, HF cache) on the CPU with the "
                     f"call pattern of the reference's HF benchmark worker: a {args.prompt}-token "
                     f"prompt in one call (untimed), then {warmup} + {steps} forced decode tokens, one "
                     f"per call with logits_to_keep=1, argmax and host read per step, contexts "
                     f"{args.prompt + 1}..{end}, {threads} threads; value_1_thread: 1 thread, "
                     f"{min(steps, 4)} tokens after 1 warm-up"}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": 1000.0 / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": workload(args) + " (HF eager on the CPU)", "model": args.config,
                   "global_batch": 1, "seq_len": args.capacity, "prompt": args.prompt,
                   "parallelism": "cpu"},
        "cpu_baseline": res,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.measure == "prefill":
        return measure_prefill(args, dist, dev, world, rank)

    from xinfer_b200 import configs, synthetic
    from xinfer_b200.engine import Engine, Runner, pack_linears

    g = configs.get(args.config)
    weights = pack_linears(g, synthetic.make_state_dict(g, seed=0, device=dev))
    eng = Engine(g, weights, capacity=args.capacity, device=dev)
    runner = Runner(eng)
    B = args.batch
    if not 1 <= B <= 8:
        raise SystemExit("--batch must be 1..8")
    if B == 1:
        lengths = [args.prompt]
    else:  # ragged rows: lengths ~ U[2, prompt] from a seed (BASELINE's batched configuration)
        gen = torch.Generator().manual_seed(4242 + rank)
        lengths = [int(x) for x in torch.randint(2, args.prompt + 1, (B,), generator=gen)]
    prompts = [synthetic.random_prompt(g, n, seed=1000 + 17 * b + rank) for b, n in enumerate(lengths)]
    if max(lengths) + args.warmup + args.steps + 1 > args.capacity:  # each leg starts from a fresh prefill
        raise SystemExit("prompt + steps exceed the KV capacity")
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def prefill_rows():
        runner.reset()
        if B == 1:  # the prompt through the prefill path (tensor-core GEMMs), 512 tokens per chunk
            runner.prefill(prompts[0])
            return
        for t in range(max(lengths)):
            runner.step_batch([[p[t]] if t < len(p) else [] for p in prompts])

    starts = list(lengths)
    total = args.warmup + args.steps

    # ---- value: device-resident greedy decode ------------------------------------------------
    prefill_rows()
    tok = [torch.zeros(B, dtype=torch.int64, device=dev) for _ in range(2)]
    tok[0].copy_(runner.next_tokens[:B])
    pos = torch.tensor([[s + k for s in starts] for k in range(total)], dtype=torch.int64, device=dev)

    def device_step(k):
        eng.launch(tok[k % 2], pos[k], [s + k + 1 for s in starts], [1] * B, runner.state, runner.state,
                   runner.logits, tok[(k + 1) % 2])

    for k in range(args.warmup):
        device_step(k)
    eng.check_device_error()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        ev0.record(stream)
        for k in range(args.warmup, total):
            device_step(k)
        ev1.record(stream)
        barrier()
    ms = ev0.elapsed_time(ev1)
    eng.check_device_error()
    ms = max_over_ranks(ms, dist, dev)
    value = job_throughput(world, B * args.steps, ms / 1000.0)
    mean_launch_s = ms / 1000.0 / args.steps

    # ---- e2e: public runner path with host buffers -------------------------------------------
    prefill_rows()
    host_in = torch.zeros(2 * B, dtype=torch.int64).pin_memory()
    host_out = torch.zeros(B, dtype=torch.int64).pin_memory()
    dev_in = torch.zeros(2 * B, dtype=torch.int64, device=dev)
    host_out.copy_(runner.next_tokens[:B])
    hin, hout = host_in.numpy(), host_out.numpy()  # views of the pinned buffers
    ids_dev, pos_dev, next_dev = dev_in[0:B], dev_in[B:2 * B], runner.next_tokens[:B]
    starts_np = hin[B:2 * B].copy()
    starts_np[:] = starts
    next_host = hout.copy()

    def e2e_step(k, tokens):
        hin[:B] = tokens
        hin[B:] = starts_np + k
        dev_in.copy_(host_in, non_blocking=True)
        eng.launch(ids_dev, pos_dev, [s + k + 1 for s in starts], [1] * B, runner.state,
                   runner.state, runner.logits, runner.next_tokens)
        host_out.copy_(next_dev, non_blocking=True)
        stream.synchronize()
        return hout.copy()

    for k in range(args.warmup):
        next_host = e2e_step(k, next_host)
    barrier()
    t0 = time.perf_counter()
    for k in range(args.warmup, total):
        next_host = e2e_step(k, next_host)
    e2e_s = time.perf_counter() - t0
    eng.check_device_error()
    barrier()
    e2e_s = max_over_ranks(e2e_s, dist, dev)
    e2e_value = job_throughput(world, B * args.steps, e2e_s)

    ctxs = [st + args.warmup + (args.steps + 1) / 2.0 for st in starts]
    ctx_mean = sum(ctxs) / B
    alg = algorithmic_bytes(g, ctxs)
    peak, peak_kind = measured_peak()
    achieved = alg / mean_launch_s / 1e9
    traffic = traffic_from_profile(g, ctx_mean) if B == 1 else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload(args), "model": args.config, "global_batch": world * B,
                   "seq_len": args.capacity, "prompt": args.prompt,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (1.5 GB of weights per step)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg, "traffic": traffic},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 16 * B, "d2h_bytes_per_step": 8 * B},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if args.trace and rank == 0:
        from xinfer_b200 import _native as nat

        # one more step after the e2e leg, at the bench's context, with the stage trace on
        buf = torch.zeros(nat.TRACE_BYTES // 8, dtype=torch.int64, device=dev)
        nat.check(nat.load().xb_debug_trace(buf.data_ptr(), nat.TRACE_BYTES))
        eng.launch([int(t) for t in next_host[:B]], [s + total for s in starts],
                   [s + total + 1 for s in starts], [1] * B, runner.state, runner.state,
                   runner.logits, runner.next_tokens)
        torch.cuda.synchronize(dev)
        nat.check(nat.load().xb_debug_trace(None, 0))
        torch.save({"trace": buf.cpu(), "ncta": torch.cuda.get_device_properties(dev).multi_processor_count,
                    "stride": nat.TRACE_STRIDE, "stages": nat.TRACE_STAGES}, args.trace)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        eng.close()
        del weights, runner
        torch.cuda.empty_cache()
        line["cpu_baseline"] = cpu_baseline(args, g)
        line["cpu_baseline"]["oracle_port"] = oracle_port_rate(args, g, args.cpu_seconds)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
