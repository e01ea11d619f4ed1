"""Stale inter-stage words never pass for fresh ones, whatever the gap between launches.

Every inter-stage value carries a 16-bit tag derived from the launch epoch and the (layer,
write) position; tags of two launches agree only when their epochs differ by a multiple of 511.
The kernel therefore clears all tagged buffers at the start of any launch that comes 256 or more
epochs after the previous clear. This test sets the epoch word by hand so that the third of
three launches carries exactly the tags of the first one, and checks (i) that the launch in
between cleared the buffers and (ii) that the third launch, which uses split-KV slots the second
one left untouched, gives bit for bit the result of the same three steps without the jump.
"""

import pytest
import torch

from xinfer_b200 import configs, synthetic
from xinfer_b200.engine import Engine

pytestmark = pytest.mark.gpu

CTL_EPOCH, CTL_SCRUBBED = 128, 160  # control words of the workspace (u32 index)
TAG_PERIOD = 511


def _engine(device):
    g = configs.get("qwen3.5-tiny")
    sd = synthetic.make_state_dict(g, seed=0, jitter=0.1)
    return g, Engine(g, {k: v.to(device) for k, v in sd.items()}, capacity=512, device=device)


def _fill(state, seed, device):
    gen = torch.Generator(device=device).manual_seed(seed)
    for t in state:
        t.copy_((torch.randn(t.shape, generator=gen, device=device) * 0.5).to(t.dtype))


def _steps(eng, g, device, jump):
    """Three launches: 400 cached positions (74 splits), 8 positions (2 splits), 400 again."""
    state = eng.allocate_state()
    _fill(state, 7, device)
    ctrl = eng.workspace.view(torch.int32)
    out = []
    for k, (pos, tok) in enumerate(((399, 11), (7, 12), (399, 13))):
        if k == 1 and jump:
            e = int(ctrl[CTL_EPOCH].item())
            ctrl[CTL_EPOCH] = e - 1 + TAG_PERIOD - 1  # next launch: first epoch + 510
        logits = torch.empty(1, g.vocab, dtype=torch.bfloat16, device=device)
        eng.launch([tok], [pos], [pos + 1], [1], state, state, logits)
        eng.check_device_error()
        if k == 1 and jump:
            assert int(ctrl[CTL_SCRUBBED].item()) == int(ctrl[CTL_EPOCH].item()) - 1, \
                "the launch after the epoch jump must clear the tagged buffers"
        out.append(logits.clone())
    return torch.cat(out), [t.clone() for t in state]


def test_epoch_jump_of_one_tag_period(cuda_device):
    g, eng = _engine(cuda_device)
    want, want_state = _steps(eng, g, cuda_device, jump=False)
    eng.workspace.zero_()
    got, got_state = _steps(eng, g, cuda_device, jump=True)
    assert torch.equal(got, want)
    for a, b in zip(got_state, want_state):
        assert torch.equal(a, b)
    eng.close()
