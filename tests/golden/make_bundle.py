"""Write a small shared-weight archive (the bundle's weights.pt) with the reference's own writer.

Usage (needs a checkout of tqxia/xinfer; the output is committed, so tests never run this):

    python tests/golden/make_bundle.py --reference <path to the xinfer checkout>

The archive holds the seeded synthetic qwen3.5-micro weights (xinfer_b200/synthetic.py, seed 0,
norm jitter 0.1) under the parameter names the reference's Qwen3.5 ModelStep exports
(`original.model.layers.N.linear_attn.block.*`, `original.model.layers.N.self_attn.original.*`,
`original.lm_head.weight` tied to the embedding). Tensors are registered with the reference's
compiler/common/weights.py `_register` (deduplicated flat storages plus view descriptors) and
saved as compile_shared saves the archive (a scripted module with one buffer per storage and
`weights.json` as an extra file); decode.json carries the `shared_weights` contract.
"""

import argparse
import json
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from xinfer_b200 import configs, synthetic  # noqa: E402

OUT = Path(__file__).resolve().parent / "bundle-qwen3.5-micro"


def exported_name(g, name):
    """ModelStep's state-dict name of an HF parameter (compiler/qwen35/model.py:154-160 and the
    adapters' wrappers)."""
    if name.startswith("model.layers."):
        i = int(name.split(".")[2])
        if g.is_delta(i):
            name = name.replace(".linear_attn.", ".linear_attn.block.")
        else:
            name = name.replace(".self_attn.", ".self_attn.original.")
    return "original." + name


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from compiler.common import weights as W
    from compiler.common.artifacts import canonical_json, json_sha256, sha256

    g = configs.get("qwen3.5-micro")
    sd = synthetic.make_state_dict(g, seed=0, jitter=0.1)
    identity = {"model": g.name, "synthetic_seed": 0, "jitter": 0.1}
    data = dict(format=2, identity=identity, identity_sha256=json_sha256(identity), entries={},
                sources={}, storages={}, tensors={})
    storages, cache = {}, {}
    for name, tensor in sd.items():
        data["sources"][exported_name(g, name)] = W._register(tensor, data, storages, cache)
    views = sorted(set(data["sources"].values()))
    data["entries"] = {kind: {"constants": {v: v for v in views}, "package_sha256": ""}
                       for kind in ("prefill", "decode")}
    archive = W._Archive(data["identity_sha256"])
    for name in sorted(storages):
        archive.register_buffer(name, storages[name])
    OUT.mkdir(parents=True, exist_ok=True)
    path = OUT / "weights.pt"
    torch.jit.save(torch.jit.script(archive), str(path), _extra_files={"weights.json": canonical_json(data)})
    contract = dict(format=2, file="weights.pt", identity=data["identity_sha256"],
                    bytes=path.stat().st_size, sha256=sha256(path))
    (OUT / "decode.json").write_text(json.dumps({"shared_weights": contract}, indent=1) + "\n")
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
