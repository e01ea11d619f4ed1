"""The prefill path (xb_prefill_step: tensor-core GEMMs, DeltaNet scan, prefix attention) and its
GEMM (xb_gemm_bf16) on the GPU.

Prefill of T tokens is ModelStep.forward with T > 1 (compiler/qwen35/model.py:162-183): the same
model as T single-token steps. It is compared with the CPU oracle run token by token on the same
prompt: the last token's logits, the fused argmax, the KV slots written, the conv window and the
recurrent state. Bounds: the north-star bar (max-abs 2e-2 widened by one bf16 ulp, cosine 0.9999,
state rel-L2 1e-2) or, where the schedule is long enough for one-ulp flips of fp32 sums to
cascade, twice the spread that the oracle shows against its own fp64-sum twin on that schedule.
"""

import ctypes
from pathlib import Path

import pytest
import torch

from oracle import qwen_step as O
from xinfer_b200 import _native as nat
from xinfer_b200 import configs, synthetic
from xinfer_b200.engine import Engine, Runner, pack_linears

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS, LOGIT_COS, STATE_REL = 2e-2, 0.9999, 1e-2
_MODELS = {}


def model(name, capacity, device):
    key = (name, capacity)
    if key not in _MODELS:
        g = configs.get(name)
        sd = synthetic.make_state_dict(g, seed=0, jitter=0.1)
        eng = Engine(g, {k: v.to(device) for k, v in sd.items()}, capacity=capacity, device=device)
        _MODELS[key] = (g, sd, O.prepare_weights(sd), eng)
    return _MODELS[key]


@pytest.mark.parametrize("m,n,k", [(1, 1024, 1024), (7, 8224, 1024), (128, 3584, 1024), (300, 1024, 3584),
                                   (512, 2048, 2560), (1, 151936, 1024), (513, 24, 64), (37, 5, 64),
                                   (512, 2, 1024), (100, 2056, 1000), (65, 1032, 4104), (1, 248320, 1024)])
def test_gemm_matches_fp32_product(m, n, k, cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device=cuda_device).manual_seed(m * 7 + n)
    x = torch.randn(m, k, generator=gen, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=gen, device=cuda_device) * 0.02).to(torch.bfloat16)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    lib = nat.load()
    nat.check(lib.xb_gemm_bf16(m, n, k, x.data_ptr(), w.data_ptr(), out.data_ptr(),
                               ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)))
    want = x.float() @ w.float().t()
    # one rounding of an fp32 sum: within one bf16 ulp of the fp32 product (plus a small absolute
    # allowance for sums that cancel)
    excess = (out.float() - want).abs() - (want.abs() * 2.0 ** -7 + 1e-3)
    assert excess.max().item() <= 0
    assert (out.float() == want.to(torch.bfloat16).float()).float().mean().item() >= 0.95


def oracle_run(g, W, prompt, capacity, dtype=torch.float32):
    state = O.allocate_state(g, capacity, rows=1)
    logits = []
    with O.accumulate(dtype):
        for pos, tok in enumerate(prompt):
            out, state = O.decode_step(g, W, [tok], [pos], state, [pos + 1], [1])
            logits.append(out[0])
    return torch.stack(logits), state


@pytest.mark.parametrize("name,T,chunks", [
    ("qwen3.5-tiny", 1, 1), ("qwen3.5-tiny", 5, 1), ("qwen3.5-tiny", 64, 1), ("qwen3.5-tiny", 200, 1),
    ("qwen3.5-tiny", 160, 2), ("qwen3-tiny", 37, 1), ("qwen3-tiny", 300, 3), ("qwen3.5-tiny-hv32", 100, 1),
    ("qwen3.5-0.8b-l4", 130, 1), ("qwen3-0.6b-l2", 512, 1)])
def test_prefill_matches_token_by_token_oracle(name, T, chunks, cuda_device):
    cap = 640
    g, sd, W, eng = model(name, cap, cuda_device)
    prompt = synthetic.random_prompt(g, T, seed=T + 11)
    state = [t.narrow(0, 0, 1) for t in eng.allocate_state()]
    logits = torch.empty(g.vocab, dtype=torch.bfloat16, device=cuda_device)
    tok = torch.empty(1, dtype=torch.int64, device=cuda_device)
    bounds = [0] + [T * (i + 1) // chunks for i in range(chunks)]
    for c0, c1 in zip(bounds[:-1], bounds[1:]):
        ids = torch.tensor(prompt[c0:c1], dtype=torch.int64, device=cuda_device)
        eng.prefill(ids, c0, state, state, logits, tok)
    eng.check_prefill_error()
    want, ostate = oracle_run(g, W, prompt, cap)
    twin, tstate = oracle_run(g, W, prompt, cap, torch.float64)
    # the oracle's own spread on this schedule over its last steps
    tail = range(max(0, T - 16), T)
    spread = max((want[s].float() - twin[s].float()).abs().max().item() for s in tail)
    cspread = max(1.0 - O.cosine(want[s], twin[s]) for s in tail)
    got = logits.float().cpu()
    ref = want[-1].float()
    excess = ((got - ref).abs() - (max(LOGIT_MAX_ABS, 2 * spread) + ref.abs() * 2.0 ** -7)).max().item()
    assert excess <= 0, f"{name} T={T}: max abs {(got - ref).abs().max().item()}"
    assert O.cosine(got, ref) >= min(LOGIT_COS, 1 - 2 * cspread)
    assert int(tok[0]) == int(torch.argmax(got))
    for i in range(g.num_layers):
        a0, a1 = state[2 * i].cpu(), state[2 * i + 1].cpu()
        b0, b1 = ostate[2 * i], ostate[2 * i + 1]
        t0, t1 = tstate[2 * i], tstate[2 * i + 1]
        if g.is_delta(i):
            pairs = ((a0.float(), b0.float(), t0.float()), (a1, b1, t1))
        else:
            pairs = ((a0[:, :, :T].float(), b0[:, :, :T].float(), t0[:, :, :T].float()),
                     (a1[:, :, :T].float(), b1[:, :, :T].float(), t1[:, :, :T].float()))
            assert torch.count_nonzero(a0[:, :, T:]) == 0 and torch.count_nonzero(a1[:, :, T:]) == 0
        for a, b, c in pairs:
            assert O.rel_l2(a, b) <= max(STATE_REL, 2 * O.rel_l2(c, b)), f"{name} T={T} state of layer {i}"


def test_packed_projections_give_the_same_prefill(cuda_device):
    """Weights in the reference's packed layout (each projection group as adjacent rows of one
    tensor) run one GEMM per group; the result equals the per-projection GEMMs bit for bit."""
    g, sd, W, eng = model("qwen3.5-0.8b-l4", 640, cuda_device)
    packed = Engine(g, pack_linears(g, {k: v.to(cuda_device) for k, v in sd.items()}), capacity=640,
                    device=cuda_device)
    prompt = torch.tensor(synthetic.random_prompt(g, 200, seed=5), dtype=torch.int64, device=cuda_device)
    outs = []
    for e in (eng, packed):
        state = [t.narrow(0, 0, 1) for t in e.allocate_state()]
        logits = torch.empty(g.vocab, dtype=torch.bfloat16, device=cuda_device)
        e.prefill(prompt, 0, state, state, logits)
        e.check_prefill_error()
        outs.append([logits] + [t.clone() for t in state])
    differ = [(i, (a.float() - b.float()).abs().max().item()) for i, (a, b) in enumerate(zip(*outs))
              if not torch.equal(a, b)]
    packed.close()
    assert not differ, f"outputs (0 = logits, then state) that differ, with max abs: {differ}"


def test_runner_prefill_then_decode_matches_decode_only(cuda_device):
    """A 300-token prompt through Runner.prefill, then greedy steps, against the same prompt fed
    one token per decode call: the same model, so the continuation agrees up to near-ties."""
    g, sd, W, eng = model("qwen3.5-tiny", 640, cuda_device)
    prompt = synthetic.random_prompt(g, 300, seed=3)
    a = Runner(eng)
    a.prefill(prompt)
    la = a.logits[0].float().cpu()
    b = Runner(eng)
    for t in prompt:
        b.step([t])
    lb = b.logits[0].float().cpu()
    assert O.cosine(la, lb) >= 0.9995 and (la - lb).abs().max().item() <= 0.1
    assert a.positions[0] == b.positions[0] == 300


GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("fixture", sorted(p.stem for p in GOLDEN.glob("*.pt") if "prefill" in p.stem))
def test_prefill_matches_reference_fixture(fixture, cuda_device):
    """The reference's own prefill chunk (its chunk-64 DeltaNet path) and the decode steps after
    it, against this library's prefill + decode: held to the north-star bar, or twice the oracle's
    spread against its fp64-sum twin on the same schedule where that is larger."""
    fx = torch.load(GOLDEN / f"{fixture}.pt", weights_only=False)
    g, sd, W, eng = model(fx["config"], fx["capacity"], cuda_device)
    assert fx["jitter"] == 0.1 and fx["seed"] == 0
    state = [t.narrow(0, 0, 1) for t in eng.allocate_state()]
    logits = torch.empty(g.vocab, dtype=torch.bfloat16, device=cuda_device)
    tok = torch.empty(1, dtype=torch.int64, device=cuda_device)
    # the oracle and its twin, token by token, for the bounds
    prompt = [t for step in fx["schedule"] for t in step[0]]
    want, _ = oracle_run(g, W, prompt, fx["capacity"])
    twin, _ = oracle_run(g, W, prompt, fx["capacity"], torch.float64)
    pos = 0
    for s, step in enumerate(fx["schedule"]):
        row = step[0]
        if len(row) > 1:
            eng.prefill(torch.tensor(row, dtype=torch.int64, device=cuda_device), pos, state, state, logits, tok)
        else:
            out = eng.decode_step(torch.tensor([[row[0]]], dtype=torch.int64, device=cuda_device),
                                  torch.tensor([[pos]], dtype=torch.int64, device=cuda_device), state,
                                  torch.tensor([pos + 1], dtype=torch.int32), torch.tensor([1], dtype=torch.int32),
                                  next_tokens=tok)
            logits.copy_(out[0][0])
            state = list(out[1:])
        pos += len(row)
        got, ref = logits.float().cpu(), fx["logits"][s, 0].float()
        spread = (want[pos - 1].float() - twin[pos - 1].float()).abs().max().item()
        bound = max(LOGIT_MAX_ABS, 2 * spread)
        assert ((got - ref).abs() - (bound + ref.abs() * 2.0 ** -7)).max().item() <= 0, (s, (got - ref).abs().max().item())
        assert O.cosine(got, ref) >= min(LOGIT_COS, 1 - 2 * (1 - O.cosine(want[pos - 1], twin[pos - 1])))
        assert int(tok[0]) == int(torch.argmax(got))
    eng.check_prefill_error()
