"""Host side of the decode megakernel: device plan, workspace, launches, and the reference's
decode ABI on top of them.

Two entry levels mirror the reference:
  * ``Engine.decode_step`` follows ``ModelStep.forward`` at T == 1
    (compiler/qwen3/model.py:70-95, compiler/qwen35/model.py:162-183): explicit tensor state,
    KV updated in place, Qwen3.5 conv / recurrent state returned as fresh replacement tensors,
    empty rows (query length 0) get zero logits and unchanged state;
  * ``Runner`` follows ``Runner<Spec>`` (runtime/common/runner.h:14-125): it owns eight state
    rows, validates requests before touching state, tracks per-row positions and runs greedy
    generation with the argmax fused into the kernel (runtime/common/generation.h:28-48).
    Its DeltaNet state is updated in place, so it needs no ``at::cat`` of untouched tail rows
    (runtime/common/state.h:64-73) and no per-step allocation.
PyTorch provides device memory and streams only; all math runs in the CUDA library.
"""

import ctypes

import torch

from . import _native as nat
from .configs import QWEN35


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def linear_groups(geometry):
    """Per layer, the HF names of the projections that read the same input, in the order the
    reference's pack_linears pass concatenates them (compiler/common/passes/pack_linears.py:22-142):
    DeltaNet in_proj qkv | z | b | a, attention q | k | v, MLP gate | up."""
    groups = []
    for i in range(geometry.num_layers):
        p = f"model.layers.{i}."
        if geometry.is_delta(i):
            groups.append([p + f"linear_attn.in_proj_{n}.weight" for n in ("qkv", "z", "b", "a")])
        else:
            groups.append([p + f"self_attn.{n}_proj.weight" for n in ("q", "k", "v")])
        groups.append([p + f"mlp.{n}_proj.weight" for n in ("gate", "up")])
    return groups


def pack_linears(geometry, weights):
    """A copy of `weights` whose projection groups (linear_groups) live as adjacent rows of one
    tensor each, the layout of the reference's packed bundle; the HF names become views. The
    prefill then runs one GEMM per group; the decode kernel streams the same rows either way."""
    out = dict(weights)
    for names in linear_groups(geometry):
        parts = [weights[n] for n in names]
        packed = torch.cat([t.reshape(t.shape[0], -1) for t in parts], dim=0)
        row = 0
        for n, t in zip(names, parts):
            out[n] = packed[row:row + t.shape[0]].view(t.shape)
            row += t.shape[0]
    return out


class Engine:
    """One model on one GPU: weight table, RoPE table, workspace."""

    def __init__(self, geometry, weights, capacity, *, state_rows=8, device=None):
        self.lib = nat.load()
        self.g = geometry
        self.capacity = int(capacity)
        self.state_rows = int(state_rows)
        self.device = torch.device(device or "cuda")
        if self.device.type != "cuda":
            raise ValueError("the decode engine runs on CUDA devices only")
        if not 1 <= self.capacity <= geometry.max_position_embeddings:
            raise ValueError("capacity must be within 1..max_position_embeddings")
        self.weights = {}
        for name, t in weights.items():
            if t.device != self.device or t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise ValueError(f"weight {name} must be a contiguous bf16 tensor on {self.device}")
            self.weights[name] = t
        g = geometry
        geo = nat.XbGeometry()
        geo.family = nat.FAMILY_QWEN35 if g.family == QWEN35 else nat.FAMILY_QWEN3
        geo.num_layers, geo.hidden, geo.intermediate, geo.vocab = (
            g.num_layers, g.hidden, g.intermediate, g.vocab)
        geo.num_q_heads, geo.num_kv_heads, geo.head_dim = g.num_q_heads, g.num_kv_heads, g.head_dim
        geo.rotary_dim = g.rotary_dim
        geo.lin_key_heads, geo.lin_value_heads = g.lin_key_heads, g.lin_value_heads
        geo.lin_head_dim, geo.conv_width = g.lin_head_dim, g.conv_width
        geo.capacity, geo.state_rows = self.capacity, self.state_rows
        geo.rms_eps, geo.rope_theta = g.rms_eps, g.rope_theta
        # RoPE inverse frequencies exactly as the HF rotary module computes them (fp32 torch).
        inv = 1.0 / (g.rope_theta ** (torch.arange(0, g.rotary_dim, 2, dtype=torch.int64).float()
                                      / g.rotary_dim))
        self._inv = (ctypes.c_float * len(inv))(*inv.tolist())
        geo.rope_inv_freq = ctypes.cast(self._inv, ctypes.POINTER(ctypes.c_float))
        for i in range(g.num_layers):
            geo.layer_kind[i] = nat.LAYER_DELTANET if g.is_delta(i) else nat.LAYER_ATTENTION
        self._geo = geo

        W = self.weights
        mw = nat.XbModelWeights()
        mw.embed = _ptr(W["model.embed_tokens.weight"])
        mw.final_norm = _ptr(W["model.norm.weight"])
        mw.lm_head = _ptr(W.get("lm_head.weight", W["model.embed_tokens.weight"]))
        for i in range(g.num_layers):
            p = f"model.layers.{i}."
            lw = mw.layers[i]
            lw.input_norm = _ptr(W[p + "input_layernorm.weight"])
            lw.post_norm = _ptr(W[p + "post_attention_layernorm.weight"])
            lw.gate = _ptr(W[p + "mlp.gate_proj.weight"])
            lw.up = _ptr(W[p + "mlp.up_proj.weight"])
            lw.down = _ptr(W[p + "mlp.down_proj.weight"])
            if g.is_delta(i):
                a = p + "linear_attn."
                lw.in_qkv = _ptr(W[a + "in_proj_qkv.weight"])
                lw.in_z = _ptr(W[a + "in_proj_z.weight"])
                lw.in_b = _ptr(W[a + "in_proj_b.weight"])
                lw.in_a = _ptr(W[a + "in_proj_a.weight"])
                lw.conv_w = _ptr(W[a + "conv1d.weight"])
                lw.a_log = _ptr(W[a + "A_log"])
                lw.dt_bias = _ptr(W[a + "dt_bias"])
                lw.gnorm = _ptr(W[a + "norm.weight"])
                lw.out_proj = _ptr(W[a + "out_proj.weight"])
            else:
                a = p + "self_attn."
                for field, key in (("q_proj", "q_proj.weight"), ("k_proj", "k_proj.weight"),
                                   ("v_proj", "v_proj.weight"), ("o_proj", "o_proj.weight"),
                                   ("q_norm", "q_norm.weight"), ("k_norm", "k_norm.weight")):
                    setattr(lw, field, _ptr(W[a + key]))
        self._mw = mw
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            nat.check(self.lib.xb_model_create(ctypes.byref(geo), ctypes.byref(mw), ctypes.byref(handle)))
        self.handle = handle
        nbytes = ctypes.c_size_t()
        nat.check(self.lib.xb_decode_workspace_bytes(handle, nat.MAX_BATCH, ctypes.byref(nbytes)))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=self.device)
        self._args = nat.XbStepArgs()
        self._ws_ptr, self._ws_bytes = self.workspace.data_ptr(), self.workspace.numel()
        self._bound_in = self._bound_out = None
        self._prefill_ws = None

    def close(self):
        if getattr(self, "handle", None):
            self.lib.xb_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- state ------------------------------------------------------------------------------
    def state_specs(self):
        """Ordered (layer, kind, shape, dtype) as the reference's state_specs / allocate_cache
        (compiler/qwen35/model.py:59-77, compiler/qwen3/model.py:29-35)."""
        g, rows = self.g, self.state_rows
        specs = []
        for i in range(g.num_layers):
            if g.is_delta(i):
                specs.append((i, "conv", (rows, g.conv_channels, g.conv_width), torch.bfloat16))
                specs.append((i, "recurrent", (rows, g.lin_value_heads, g.lin_head_dim, g.lin_head_dim),
                              torch.float32))
            else:
                kv = (rows, g.num_kv_heads, self.capacity, g.head_dim)
                specs.append((i, "key", kv, torch.bfloat16))
                specs.append((i, "value", kv, torch.bfloat16))
        return specs

    def allocate_state(self, fill=0.0):
        return [torch.full(shape, fill if kind in ("key", "value") else 0.0, dtype=dt, device=self.device)
                for _, kind, shape, dt in self.state_specs()]

    # -- launch -----------------------------------------------------------------------------
    def launch(self, input_ids, cache_position, kv_lengths, query_lengths, state_in, state_out,
               logits, next_tokens=None, stream=None):
        """One decode step. state_in / state_out: per-spec tensors addressing row 0 (state_out
        entries for KV are the same tensors as state_in)."""
        B = len(kv_lengths)
        a = self._args
        a.batch = B
        if isinstance(input_ids, torch.Tensor):
            a.input_ids = input_ids.data_ptr()
            a.cache_position = cache_position.data_ptr()
        else:  # host values travel as launch parameters
            a.input_ids = a.cache_position = None
            for b in range(B):
                a.host_ids[b] = int(input_ids[b])
                a.host_positions[b] = int(cache_position[b])
        for b in range(B):
            a.kv_lengths[b] = int(kv_lengths[b])
            a.query_lengths[b] = int(query_lengths[b])
        if state_in is not self._bound_in or state_out is not self._bound_out:
            self._bind(state_in, state_out)
        a.logits = logits.data_ptr()
        a.next_tokens = next_tokens.data_ptr() if next_tokens is not None else None
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        nat.check(self.lib.xb_decode_step(self.handle, ctypes.byref(a), self._ws_ptr, self._ws_bytes,
                                          ctypes.c_void_p(st.cuda_stream)))

    def _bind(self, state_in, state_out):
        """Per-layer state pointers of the launch arguments. They are kept for the next launch
        with the same two list objects (a decode loop passes its state lists unchanged), so a
        caller that replaces tensors inside a list must pass a new list."""
        a = self._args
        for i in range(self.g.num_layers):
            ls = a.layers[i]
            s0, s1 = state_in[2 * i], state_in[2 * i + 1]
            if self.g.is_delta(i):
                o0, o1 = state_out[2 * i], state_out[2 * i + 1]
                ls.conv_in, ls.rec_in = s0.data_ptr(), s1.data_ptr()
                ls.conv_out, ls.rec_out = o0.data_ptr(), o1.data_ptr()
                ls.k_cache = ls.v_cache = None
            else:
                ls.k_cache, ls.v_cache = s0.data_ptr(), s1.data_ptr()
                ls.conv_in = ls.rec_in = ls.conv_out = ls.rec_out = None
        self._bound_in, self._bound_out = state_in, state_out

    # -- prefill ----------------------------------------------------------------------------
    def prefill(self, input_ids, start_position, state_in, state_out, logits, next_token=None,
                stream=None):
        """ModelStep.forward with T > 1 for one row (compiler/qwen35/model.py:162-183):
        input_ids CUDA int64 [T] (1..512 tokens) at cache positions start_position..+T-1 of state
        row 0; KV appended in place, DeltaNet state read from state_in and written to state_out
        (the same list updates in place); logits of the last token into `logits` (bf16 [vocab]),
        its argmax into `next_token` (int64 [1]) when given."""
        T = int(input_ids.numel())
        if not 1 <= T <= 512:
            raise ValueError("prefill takes 1..512 tokens")
        if input_ids.dtype != torch.int64 or input_ids.device != self.device or not input_ids.is_contiguous():
            raise ValueError("input_ids must be a contiguous CUDA int64 tensor")
        if self._prefill_ws is None:
            nbytes = ctypes.c_size_t()
            nat.check(self.lib.xb_prefill_workspace_bytes(self.handle, 512, ctypes.byref(nbytes)))
            self._prefill_ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=self.device)
        a = nat.XbPrefillArgs()
        a.tokens = T
        a.input_ids = input_ids.data_ptr()
        a.start_position = int(start_position)
        for i in range(self.g.num_layers):
            ls = a.layers[i]
            s0, s1 = state_in[2 * i], state_in[2 * i + 1]
            if self.g.is_delta(i):
                o0, o1 = state_out[2 * i], state_out[2 * i + 1]
                ls.conv_in, ls.rec_in = s0.data_ptr(), s1.data_ptr()
                ls.conv_out, ls.rec_out = o0.data_ptr(), o1.data_ptr()
            else:
                ls.k_cache, ls.v_cache = s0.data_ptr(), s1.data_ptr()
        a.logits = logits.data_ptr()
        a.next_token = next_token.data_ptr() if next_token is not None else None
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        nat.check(self.lib.xb_prefill_step(self.handle, ctypes.byref(a), self._prefill_ws.data_ptr(),
                                           self._prefill_ws.numel(), ctypes.c_void_p(st.cuda_stream)))

    def check_prefill_error(self, stream=None):
        if self._prefill_ws is None:
            return
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        err = ctypes.c_int32()
        nat.check(self.lib.xb_workspace_check(self._prefill_ws.data_ptr(), ctypes.c_void_p(st.cuda_stream),
                                              ctypes.byref(err)))

    def check_device_error(self, stream=None):
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        err = ctypes.c_int32()
        nat.check(self.lib.xb_workspace_check(self.workspace.data_ptr(), ctypes.c_void_p(st.cuda_stream),
                                              ctypes.byref(err)))

    # -- reference decode ABI ---------------------------------------------------------------
    def decode_step(self, input_ids, cache_position, state, kv_lengths, query_lengths, *,
                    next_tokens=None):
        """ModelStep.forward at T == 1 with the reference's tensor contract."""
        g = self.g
        if input_ids.dim() != 2 or input_ids.shape[1] != 1:
            raise ValueError("decode expects input_ids [B, 1]")
        B = input_ids.shape[0]
        if not 1 <= B <= min(nat.MAX_BATCH, self.state_rows):
            raise ValueError("batch must be 1..8")
        for t, name in ((input_ids, "input_ids"), (cache_position, "cache_position")):
            if t.shape != (B, 1) or t.dtype != torch.int64 or t.device != self.device:
                raise ValueError(f"{name} must be CUDA int64 [B, 1]")
        for t in (kv_lengths, query_lengths):
            if t.device.type != "cpu" or t.dtype != torch.int32 or t.shape != (B,):
                raise ValueError("kv_lengths / query_lengths must be CPU int32 [B]")
        if len(state) != 2 * g.num_layers:
            raise ValueError("incorrect state count")
        specs = self.state_specs()
        for t, (_, kind, shape, dt) in zip(state, specs):
            if t.shape != (B,) + tuple(shape[1:]) or t.dtype != dt or t.device != self.device \
                    or not t.is_contiguous():
                raise ValueError(f"incorrect {kind} state shape/dtype/device/layout")
        out_state = list(state)
        for i in range(g.num_layers):
            if g.is_delta(i):
                out_state[2 * i] = torch.empty_like(state[2 * i])
                out_state[2 * i + 1] = torch.empty_like(state[2 * i + 1])
        logits = torch.empty((B, g.vocab), dtype=torch.bfloat16, device=self.device)
        ids = input_ids.contiguous().view(B)
        pos = cache_position.contiguous().view(B)
        self.launch(ids, pos, kv_lengths.tolist(), query_lengths.tolist(), state, out_state,
                    logits, next_tokens)
        if g.family == QWEN35:
            return (logits, *out_state)
        return logits


class Runner:
    """Greedy decode runner over eight caller-owned state rows (runtime/common/runner.h)."""

    def __init__(self, engine, *, eos=()):
        self.engine = engine
        self.g = engine.g
        self.state = engine.allocate_state()
        dev = engine.device
        self.logits = torch.empty((nat.MAX_BATCH, self.g.vocab), dtype=torch.bfloat16, device=dev)
        self.next_tokens = torch.zeros(nat.MAX_BATCH, dtype=torch.int64, device=dev)
        self._tok_host = torch.zeros(nat.MAX_BATCH, dtype=torch.int64).pin_memory()
        self.eos = set(eos)
        self.reset()

    def reset(self, fill=0.0):
        """KV rows refilled with `fill`, functional state zeroed (runtime/common/state.h:21-37)."""
        for (_, kind, _, _), t in zip(self.engine.state_specs(), self.state):
            t.fill_(fill if kind in ("key", "value") else 0.0)
        self.positions = [0] * self.engine.state_rows
        self.decode_calls = 0

    def step_batch(self, rows):
        """One decode call; rows[b] is [] (empty row) or [token]. Returns logits [B, vocab]."""
        B = len(rows)
        if not 1 <= B <= self.engine.state_rows:
            raise ValueError("batch must be 1..8")
        if any(len(r) > 1 for r in rows):
            raise ValueError("the decode runner takes at most one token per row")
        if not any(rows):
            raise ValueError("at least one row must be active")
        for b, r in enumerate(rows):
            if len(r) > self.engine.capacity - self.positions[b]:
                raise ValueError("Context capacity exceeded")
            if self.positions[b] + len(r) == 0:
                raise ValueError("Each row must start with tokens")
            for t in r:
                if not 0 <= t < self.g.vocab:
                    raise ValueError("token id out of range")
        ids = [r[0] if r else 0 for r in rows]
        pos = [self.positions[b] for b in range(B)]
        kv = [self.positions[b] + len(rows[b]) for b in range(B)]
        q = [len(r) for r in rows]
        # token ids and positions travel as launch parameters: no host-to-device copy
        self.engine.launch(ids, pos, kv, q, self.state, self.state, self.logits, self.next_tokens)
        for b in range(B):
            self.positions[b] += len(rows[b])
        self.decode_calls += 1
        return self.logits[:B]

    def step(self, tokens):
        return self.step_batch([list(tokens)])

    def prefill(self, prompt):
        """Row 0's prompt through the prefill path in chunks of up to 512 tokens (the reference
        runner's prefill.pt2 calls, runtime/common/runner.h:30-78); the last token's logits and
        greedy token land in logits[0] / next_tokens[0]."""
        if len(prompt) > self.engine.capacity - self.positions[0]:
            raise ValueError("Context capacity exceeded")
        if self.positions[0] + len(prompt) == 0:
            raise ValueError("Each row must start with tokens")
        for t in prompt:
            if not 0 <= t < self.g.vocab:
                raise ValueError("token id out of range")
        dev = self.engine.device
        for c0 in range(0, len(prompt), 512):
            chunk = torch.tensor(prompt[c0:c0 + 512], dtype=torch.int64).to(dev)
            self.engine.prefill(chunk, self.positions[0], self.state, self.state, self.logits[0],
                                self.next_tokens[:1])
            self.positions[0] += chunk.numel()
        self.decode_calls += 1
        return self.logits[:1]

    def next_token(self, row=0):
        self._tok_host.copy_(self.next_tokens)
        torch.cuda.current_stream(self.engine.device).synchronize()
        return int(self._tok_host[row])

    def generate(self, prompt, limit):
        """Greedy generation (runtime/common/generation.h:28-48); argmax fused in the kernel."""
        if len(prompt) + limit > self.engine.capacity:
            raise ValueError("Context capacity exceeded")
        self.prefill(prompt)
        out = []
        for _ in range(limit):
            tok = self.next_token()
            out.append(tok)
            if tok in self.eos or len(out) == limit:
                break
            self.step([tok])
        return out
