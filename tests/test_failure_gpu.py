"""Failure detection of the decode kernel: bounded waits end a launch with an error status.

The reference reports failures through the runner's exceptions (runtime/common/runner.h); on the
device it has no equivalent. Here every wait of the persistent kernel is bounded: a stage whose
inputs never appear makes the launch give up, every CTA returns, the workspace holds the error
code and the CUDA context stays usable. The failure is injected on the host's request
(xb_debug_fault: CTA 0 withholds one stage's outputs, the wait limit is shortened); nothing
faults, traps or hangs the GPU.
"""

import ctypes

import pytest
import torch

from xinfer_b200 import _native as nat
from xinfer_b200 import configs, synthetic
from xinfer_b200.engine import Engine

DERR_WAIT = 1


def one_step(eng, state, dev):
    ids = torch.tensor([[7]], dtype=torch.int64, device=dev)
    pos = torch.tensor([[3]], dtype=torch.int64, device=dev)
    out = eng.decode_step(ids, pos, state, torch.tensor([4], dtype=torch.int32),
                          torch.tensor([1], dtype=torch.int32))
    return out[0].clone()


@pytest.mark.gpu
@pytest.mark.parametrize("withhold", [0, 2])
def test_withheld_stage_times_out_and_context_recovers(withhold, cuda_device):
    g = configs.get("qwen3.5-tiny")
    W = synthetic.make_state_dict(g, seed=5, device=cuda_device)
    eng = Engine(g, W, capacity=16, device=cuda_device)
    full = eng.allocate_state()
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    for t in full:
        t.copy_(torch.randn(t.shape, generator=gen, device=cuda_device).to(t.dtype) * 0.1)
    state = [t.narrow(0, 0, 1) for t in full]
    lib = nat.load()

    good = one_step(eng, state, cuda_device)
    eng.check_device_error()

    nat.check(lib.xb_debug_fault(withhold, 20_000_000))  # stage `withhold` withheld, 20 ms waits
    try:
        one_step(eng, state, cuda_device)
        stream = torch.cuda.current_stream(cuda_device)
        code = ctypes.c_int32()
        rc = lib.xb_workspace_check(eng.workspace.data_ptr(), ctypes.c_void_p(stream.cuda_stream),
                                    ctypes.byref(code))
    finally:
        nat.check(lib.xb_debug_fault(-1, 0))
    assert rc == nat.XB_ERR_DEVICE, "a withheld stage must end the launch with a device error"
    assert code.value == DERR_WAIT

    # the context and the workspace are usable again, and the same step gives the same logits
    again = one_step(eng, state, cuda_device)
    eng.check_device_error()
    assert torch.equal(again, good)


@pytest.mark.gpu
def test_fault_knob_rejects_tiny_limits(cuda_device):
    lib = nat.load()
    assert lib.xb_debug_fault(0, 1000) == nat.XB_ERR_INVALID
    nat.check(lib.xb_debug_fault(-1, 0))
