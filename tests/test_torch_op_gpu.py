"""The torch operators (and their AOTInductor C shim) against Engine.decode_step: the same
kernel behind two entry points, so logits and replacement state must agree bit for bit."""

import ctypes

import pytest
import torch

from xinfer_b200 import configs, synthetic, torch_ops
from xinfer_b200.engine import Engine

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


pytestmark = pytest.mark.gpu


def _setup(name, device, capacity=16):
    g = configs.get(name)
    sd = {k: v.to(device) for k, v in synthetic.make_state_dict(g, seed=0, jitter=0.1).items()}
    return g, sd, Engine(g, sd, capacity=capacity, device=device), torch_ops.DecodeStep(g, sd, capacity)


def _steps(fn, eng, rows, device, steps=4):
    full = eng.allocate_state()
    state = [t.narrow(0, 0, rows) for t in full]
    gen = torch.Generator().manual_seed(5)
    out = []
    for pos in range(steps):
        ids = torch.randint(0, eng.g.vocab, (rows, 1), generator=gen).to(device)
        cp = torch.full((rows, 1), pos, dtype=torch.int64, device=device)
        res = fn(ids, cp, state, torch.full((rows,), pos + 1, dtype=torch.int32),
                 torch.ones(rows, dtype=torch.int32))
        if isinstance(res, tuple):
            logits, *state = res
        else:
            logits = res
        out.append(logits.clone())
    torch.cuda.synchronize(device)
    return torch.stack(out), [t.clone() for t in state]


@pytest.mark.parametrize("name,rows", [("qwen3.5-tiny", 1), ("qwen3.5-tiny", 4), ("qwen3-tiny", 2)])
def test_operator_matches_engine(name, rows, cuda_device):
    g, sd, eng, op = _setup(name, cuda_device)
    want, wstate = _steps(eng.decode_step, eng, rows, cuda_device)
    got, gstate = _steps(op, eng, rows, cuda_device)
    assert torch.equal(got, want)
    for a, b in zip(gstate, wstate):
        assert torch.equal(a, b)
    eng.close()


def test_operator_on_a_side_stream(cuda_device):
    g, sd, eng, op = _setup("qwen3.5-tiny", cuda_device)
    want, _ = _steps(op, eng, 1, cuda_device)
    side = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(side):
        got, _ = _steps(op, eng, 1, cuda_device)
    side.synchronize()
    assert torch.equal(got, want)
    eng.close()


def test_aoti_shim_matches_operator(cuda_device):
    g, sd, eng, op = _setup("qwen3.5-tiny", cuda_device)
    lib = ctypes.CDLL(str(torch_ops.LIBRARY))
    shim = lib.aoti_torch_cuda_qwen35_decode_step
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    shim.restype = ctypes.c_int32
    shim.argtypes = [vp, vp, ctypes.POINTER(vp), i64, vp, vp, ctypes.POINTER(vp), i64,
                     ctypes.POINTER(i64), i64, ctypes.POINTER(ctypes.c_double), i64, ctypes.POINTER(vp), i64]
    state = [t.narrow(0, 0, 1) for t in eng.allocate_state()]
    ids = torch.tensor([[7]], dtype=torch.int64, device=cuda_device)
    cp = torch.zeros((1, 1), dtype=torch.int64, device=cuda_device)
    kv, q = torch.ones(1, dtype=torch.int32), torch.ones(1, dtype=torch.int32)
    want = op(ids, cp, [t.clone() for t in state], kv, q)
    ins, c_ins = new_handles([ids, cp, kv, q])
    st, c_st = new_handles(state)
    ws, c_ws = new_handles(op.weights)
    n_out = 1 + 2 * sum(g.is_delta(i) for i in range(g.num_layers))
    outs = (vp * n_out)()
    try:
        rc = shim(ins[0], ins[1], (vp * len(st))(*st), len(st), ins[2], ins[3], (vp * len(ws))(*ws),
                  len(ws), (i64 * len(op.geometry))(*op.geometry), len(op.geometry),
                  (ctypes.c_double * 2)(*op.params), 2, outs, n_out)
        assert rc == 0
        got = steal([outs[i] for i in range(n_out)])
    finally:
        torch._C._aoti.alloc_tensors_by_stealing_from_void_ptrs(c_ins + c_st + c_ws)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(got[0], want[0])
    k = 1
    for i in range(g.num_layers):
        if g.is_delta(i):
            assert torch.equal(got[k], want[1 + 2 * i]) and torch.equal(got[k + 1], want[2 + 2 * i])
            k += 2
    eng.close()
