"""CPU checks of the torch operator boundary (no kernel launches): the operator library loads,
its schemas carry the ModelStep contract with the KV state marked as appended in place, the fake
kernels give the output metadata an exported graph needs, and the AOTInductor C shims convert a
rejected call into an error code instead of an exception crossing the C boundary."""

import ctypes

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from xinfer_b200 import configs, torch_ops

def _capsule_api():
    api = ctypes.pythonapi
    api.PyCapsule_GetPointer.restype = ctypes.c_void_p
    api.PyCapsule_GetPointer.argtypes = [ctypes.py_object, ctypes.c_char_p]
    api.PyCapsule_New.restype = ctypes.py_object
    api.PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
    return api


def new_handles(tensors):
    """AtenTensorHandles (new references) of tensors, as integer addresses, and their capsules."""
    caps = torch._C._aoti.unsafe_alloc_void_ptrs_from_tensors(list(tensors))
    api = _capsule_api()
    return [api.PyCapsule_GetPointer(c, None) for c in caps], caps


def steal(addresses):
    """Tensors owning the handles at these addresses (the handles are released)."""
    api = _capsule_api()
    return torch._C._aoti.alloc_tensors_by_stealing_from_void_ptrs(
        [api.PyCapsule_New(a, None, None) for a in addresses])



@pytest.fixture(scope="module")
def ops():
    torch_ops.load()
    return torch.ops.xinfer


def test_schemas(ops):
    for name, ret in (("qwen35_decode_step", "Tensor[]"), ("qwen3_decode_step", "Tensor")):
        schema = str(getattr(ops, name).default._schema)
        assert schema == (f"xinfer::{name}(Tensor input_ids, Tensor cache_position, Tensor(a!)[] state, "
                          f"Tensor kv_lengths, Tensor query_lengths, Tensor[] weights, int[] geometry, "
                          f"float[] params) -> {ret}")


def test_attention_schemas(ops):
    """The reference's schemas and tags (compiler/common/kernels/attention.cpp:128-135)."""
    assert str(ops.batched_flash_attention.default._schema) == (
        "xinfer::batched_flash_attention(Tensor q, Tensor k, Tensor v, Tensor offsets, "
        "Tensor cuda_offsets, Tensor blocks, float scale) -> Tensor")
    assert str(ops.flash_attention.default._schema) == (
        "xinfer::flash_attention(Tensor q, Tensor k, Tensor v, Tensor kv_extent, float scale) -> Tensor")
    for op in (ops.batched_flash_attention.default, ops.flash_attention.default):
        assert torch.Tag.flexible_layout in op.tags
    with FakeTensorMode():
        q = torch.empty(2, 16, 5, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(2, 8, 64, 128, dtype=torch.bfloat16, device="cuda")
        out = ops.flash_attention(q, k, k, torch.empty(9, dtype=torch.uint8), 128 ** -0.5)
        assert out.shape == q.shape and out.is_contiguous()


def _fake_args(g, batch, capacity):
    geometry, params = torch_ops.geometry_args(g, capacity)
    ids = torch.zeros((batch, 1), dtype=torch.int64, device="cuda")
    state = []
    for i in range(g.num_layers):
        if g.is_delta(i):
            state.append(torch.empty((batch, g.conv_channels, g.conv_width), dtype=torch.bfloat16, device="cuda"))
            state.append(torch.empty((batch, g.lin_value_heads, 128, 128), dtype=torch.float32, device="cuda"))
        else:
            kv = (batch, g.num_kv_heads, capacity, g.head_dim)
            state += [torch.empty(kv, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    lengths = torch.ones(batch, dtype=torch.int32)
    return ids, ids.clone(), state, lengths, lengths.clone(), [], geometry, params


def test_fake_kernels(ops):
    with FakeTensorMode():
        g = configs.QWEN35_0_8B
        out = ops.qwen35_decode_step(*_fake_args(g, 3, 64))
        n_delta = sum(g.is_delta(i) for i in range(g.num_layers))
        assert len(out) == 1 + 2 * n_delta
        assert out[0].shape == (3, g.vocab) and out[0].dtype == torch.bfloat16
        assert out[1].shape == (3, g.conv_channels, 4) and out[2].shape == (3, 16, 128, 128)
        assert out[2].dtype == torch.float32
        g3 = configs.QWEN3_0_6B
        logits = ops.qwen3_decode_step(*_fake_args(g3, 2, 32))
        assert logits.shape == (2, g3.vocab) and logits.device.type == "cuda"


def test_weight_list_order():
    from xinfer_b200 import synthetic

    g = configs.QWEN35_TINY
    sd = synthetic.make_state_dict(g, seed=0)
    w = torch_ops.weight_list(g, sd)
    n_delta = sum(g.is_delta(i) for i in range(g.num_layers))
    assert len(w) == 3 + 14 * n_delta + 11 * (g.num_layers - n_delta)
    assert w[0] is sd["model.embed_tokens.weight"] and w[3] is sd["model.layers.0.input_layernorm.weight"]
    assert w[8] is sd["model.layers.0.linear_attn.in_proj_qkv.weight"]


def test_aoti_shim_reports_errors_as_codes(ops):
    """A call with CPU token ids is rejected by the operator's checks; the shim must return a
    nonzero AOTITorchError and leave its output handle untouched."""
    lib = ctypes.CDLL(str(torch_ops.LIBRARY))
    shim = lib.aoti_torch_cuda_qwen3_decode_step
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    shim.restype = ctypes.c_int32
    shim.argtypes = [vp, vp, ctypes.POINTER(vp), i64, vp, vp, ctypes.POINTER(vp), i64,
                     ctypes.POINTER(i64), i64, ctypes.POINTER(ctypes.c_double), i64, ctypes.POINTER(vp)]
    g = configs.QWEN3_TINY
    geometry, params = torch_ops.geometry_args(g, 16)
    ids = torch.zeros((1, 1), dtype=torch.int64)
    lengths = torch.ones(1, dtype=torch.int32)
    tensors = [ids, ids.clone(), lengths, lengths.clone()]
    handles, caps = new_handles(tensors)
    try:
        geo = (i64 * len(geometry))(*geometry)
        par = (ctypes.c_double * 2)(*params)
        out = vp(0)
        rc = shim(handles[0], handles[1], None, 0, handles[2], handles[3], None, 0, geo, len(geometry),
                  par, 2, ctypes.byref(out))
        assert rc != 0 and out.value is None
    finally:
        torch._C._aoti.alloc_tensors_by_stealing_from_void_ptrs(caps)
