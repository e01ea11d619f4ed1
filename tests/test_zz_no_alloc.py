"""The allocation-free decode entry point (xb_decode_step_static) against the regular one.

xb_decode_step_static serves callers that cannot allocate device memory while they step the
model (a runtime that has reserved HBM for its own pool at start-up, a fixed memory plan): it keeps its scratch in a static device array instead of a caller
workspace. This test drives both entry points through the C ABI on identical inputs for two
calls in a row and compares logits and greedy tokens with the tolerance of the other parity
tests. It sits in its own file, collected last, and builds everything it needs itself.
"""

import ctypes

import pytest
import torch

from oracle import qwen_step as O
from xinfer_b200 import _native as nat
from xinfer_b200 import configs, synthetic
from xinfer_b200.engine import Engine

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999


def _args(eng, token, position, kv_len, state, logits, next_tokens):
    a = nat.XbStepArgs()
    a.batch = 1
    a.input_ids = a.cache_position = None
    a.host_ids[0] = token
    a.host_positions[0] = position
    a.kv_lengths[0] = kv_len
    a.query_lengths[0] = 1
    for i in range(eng.g.num_layers):
        ls = a.layers[i]
        s0, s1 = state[2 * i], state[2 * i + 1]
        if eng.g.is_delta(i):
            ls.conv_in = ls.conv_out = s0.data_ptr()
            ls.rec_in = ls.rec_out = s1.data_ptr()
        else:
            ls.k_cache, ls.v_cache = s0.data_ptr(), s1.data_ptr()
    a.logits = logits.data_ptr()
    a.next_tokens = next_tokens.data_ptr()
    return a


def test_static_entry_point_matches_workspace_entry_point(cuda_device):
    lib = nat.load()
    g = configs.get("qwen3.5-tiny")
    sd = synthetic.make_state_dict(g, seed=0, jitter=0.1)
    eng = Engine(g, {k: v.to(cuda_device) for k, v in sd.items()}, capacity=16, device=cuda_device)
    state_ref = eng.allocate_state()
    state_new = eng.allocate_state()
    stream = torch.cuda.current_stream(cuda_device)
    for step, token in enumerate((101, 733)):
        logits_ref = torch.empty(1, g.vocab, dtype=torch.bfloat16, device=cuda_device)
        logits_new = torch.full((1, g.vocab), 7.0, dtype=torch.bfloat16, device=cuda_device)
        tok_ref = torch.empty(1, dtype=torch.int64, device=cuda_device)
        tok_new = torch.full((1,), -1, dtype=torch.int64, device=cuda_device)
        eng.launch([token], [step], [step + 1], [1], state_ref, state_ref, logits_ref, tok_ref)
        eng.check_device_error()
        args = _args(eng, token, step, step + 1, state_new, logits_new, tok_new)
        err = ctypes.c_int32(-1)
        nat.check(lib.xb_decode_step_static(ctypes.byref(eng._geo), ctypes.byref(eng._mw),
                                            ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream),
                                            ctypes.byref(err)))
        assert err.value == 0
        torch.cuda.synchronize(cuda_device)
        got, want = logits_new[0].float().cpu(), logits_ref[0].float().cpu()
        diff = (got - want).abs().max().item()
        assert diff <= LOGIT_MAX_ABS and O.cosine(got, want) >= LOGIT_COS, (step, diff)
        assert int(tok_new[0]) == int(tok_ref[0]), step
        for a, b in zip(state_new, state_ref):
            assert O.rel_l2(a.float(), b.float()) <= 1e-2
    eng.close()


def test_static_entry_point_rejects_oversize_scratch(cuda_device):
    lib = nat.load()
    g = configs.QWEN35_4B
    geo = nat.XbGeometry()
    geo.family = nat.FAMILY_QWEN35
    geo.num_layers, geo.hidden, geo.intermediate, geo.vocab = g.num_layers, g.hidden, g.intermediate, g.vocab
    geo.num_q_heads, geo.num_kv_heads, geo.head_dim, geo.rotary_dim = 16, 4, 256, 64
    geo.lin_key_heads, geo.lin_value_heads, geo.lin_head_dim, geo.conv_width = 16, 32, 128, 4
    geo.capacity, geo.state_rows, geo.rms_eps, geo.rope_theta = 4096, 8, 1e-6, 1e4
    for i in range(g.num_layers):
        geo.layer_kind[i] = nat.LAYER_DELTANET if g.is_delta(i) else nat.LAYER_ATTENTION
    args = nat.XbStepArgs()
    args.batch = 8
    rc = lib.xb_decode_step_static(ctypes.byref(geo), ctypes.byref(nat.XbModelWeights()),
                                   ctypes.byref(args), None, None)
    assert rc == nat.XB_ERR_INVALID
    assert b"static array" in lib.xb_last_error()
