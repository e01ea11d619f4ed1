"""Loading a reference bundle's shared-weight archive (weights.pt, format 2) into the engine.

The fixture tests/golden/bundle-qwen3.5-micro was written by the reference's own archive writer
(compiler/common/weights.py, through tests/golden/make_bundle.py) from the seeded synthetic
weights under the reference's exported ModelStep names."""

import json
import shutil

import pytest
import torch

from xinfer_b200 import bundle, configs, synthetic

from conftest import ROOT

FIXTURE = ROOT / "tests" / "golden" / "bundle-qwen3.5-micro"


def test_exported_names_map_to_hf_names():
    assert bundle.hf_name("original.model.layers.0.linear_attn.block.in_proj_qkv.weight") == \
        "model.layers.0.linear_attn.in_proj_qkv.weight"
    assert bundle.hf_name("original.model.layers.3.self_attn.original.q_norm.weight") == \
        "model.layers.3.self_attn.q_norm.weight"
    assert bundle.hf_name("model.model.layers.5.self_attn.original.o_proj.weight") == \
        "model.layers.5.self_attn.o_proj.weight"
    assert bundle.hf_name("original.lm_head.weight") == "lm_head.weight"


def test_archive_round_trips_the_weights():
    g = configs.get("qwen3.5-micro")
    got = bundle.load_weights(FIXTURE)
    want = synthetic.make_state_dict(g, seed=0, jitter=0.1)
    assert set(got) == set(want)
    for name, t in want.items():
        assert got[name].dtype == t.dtype and torch.equal(got[name], t), name
    # the tied lm_head is a view of the embedding's storage, as in the archive
    assert got["lm_head.weight"].untyped_storage().data_ptr() == \
        got["model.embed_tokens.weight"].untyped_storage().data_ptr()
    ew = bundle.engine_weights(g, got)
    assert ew["lm_head.weight"].data_ptr() == ew["model.embed_tokens.weight"].data_ptr()


def test_contract_is_checked(tmp_path):
    work = tmp_path / "bundle"
    shutil.copytree(FIXTURE, work)
    meta = json.loads((work / "decode.json").read_text())
    meta["shared_weights"]["sha256"] = "0" * 64
    (work / "decode.json").write_text(json.dumps(meta))
    with pytest.raises(ValueError, match="checksum mismatch"):
        bundle.load_weights(work)
    meta["shared_weights"]["format"] = 1
    (work / "decode.json").write_text(json.dumps(meta))
    with pytest.raises(ValueError, match="Shared weights metadata is required"):
        bundle.load_weights(work)


@pytest.mark.gpu
def test_engine_from_bundle_steps_like_engine_from_state_dict(cuda_device):
    from xinfer_b200.engine import Engine

    g = configs.get("qwen3.5-micro")
    loaded = bundle.engine_weights(g, bundle.load_weights(FIXTURE, device=cuda_device))
    direct = {k: v.to(cuda_device) for k, v in synthetic.make_state_dict(g, seed=0, jitter=0.1).items()}
    outs = []
    for weights in (loaded, direct):
        eng = Engine(g, weights, capacity=32, device=cuda_device)
        state = [t.narrow(0, 0, 1) for t in eng.allocate_state()]
        logits = torch.empty(g.vocab, dtype=torch.bfloat16, device=cuda_device)
        eng.prefill(torch.arange(5, dtype=torch.int64, device=cuda_device) * 7, 0, state, state, logits)
        out = eng.decode_step(torch.tensor([[3]], device=cuda_device), torch.tensor([[5]], device=cuda_device),
                              state, torch.tensor([6], dtype=torch.int32), torch.tensor([1], dtype=torch.int32))
        torch.cuda.synchronize(cuda_device)
        outs.append((logits.clone(), out[0].clone()))
        eng.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
