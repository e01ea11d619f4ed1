"""Load the model weights of a reference bundle (the five-file bundle: prefill.pt2, decode.pt2,
weights.pt, prefill.json, decode.json; README.md:30-33) into this library's engine.

The bundle's weights live in `weights.pt`, the shared-weight archive written by
compiler/common/weights.py:294-380 (format 2, docs/package-metadata.md "Shared-weight archive and
ownership"): a TorchScript module whose buffers are deduplicated flat storages named `w_<sha256>`,
with an embedded `extra/weights.json` that maps every exported parameter name (`sources`) to a
view descriptor (storage, dtype, device, shape, stride, offset). The exported names are those of
the reference's ModelStep: its HF model under `original.` (Qwen3.5) or `model.` (Qwen3), with the
adapters' wrapper modules in the path (`linear_attn.block.`, `self_attn.original.`;
compiler/qwen35/adapters/delta.py:70-74, compiler/qwen35/adapters/attention.py:66-76). Removing
the ModelStep prefix and the wrapper segments gives the HF names this library's Engine takes.

The archive and the sidecar are checked the way the reference's reader checks them
(compiler/common/weights.py:37-104, runtime/common/spec.h): format 2, file name, byte size and
SHA-256 of weights.pt against the sidecar's `shared_weights` contract, identity digest, storage
dtype and size. Views keep sharing their storage (a tied lm_head stays the embedding).
"""

import hashlib
import json
import zipfile
from pathlib import Path

import torch

from . import synthetic

_WRAPPERS = (".block.", ".original.")


def hf_name(exported):
    """HF parameter name of an exported ModelStep parameter name."""
    for prefix in ("original.", "model."):
        if exported.startswith(prefix) and (exported[len(prefix):].startswith("model.") or
                                            exported[len(prefix):].startswith("lm_head.")):
            exported = exported[len(prefix):]
            break
    for w in _WRAPPERS:
        exported = exported.replace(w, ".")
    return exported


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _canonical_sha256(value):
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def read_manifest(archive_path):
    """The embedded extra/weights.json of a shared-weight archive (format 2)."""
    with zipfile.ZipFile(archive_path) as z:
        records = [n for n in z.namelist() if n.endswith("/extra/weights.json")]
        if len(records) != 1:
            raise ValueError("Shared weights archive metadata is missing")
        data = json.loads(z.read(records[0]))
    if not isinstance(data, dict) or data.get("format") != 2:
        raise ValueError("Shared weights archive metadata has unsupported format")
    if data.get("identity_sha256") != _canonical_sha256(data.get("identity")):
        raise ValueError("Shared weights identity mismatch")
    return data


def check_contract(directory, contract):
    """The sidecar's `shared_weights` contract against weights.pt (size, SHA-256, identity)."""
    path = Path(directory) / "weights.pt"
    if not (isinstance(contract, dict) and contract.get("format") == 2 and contract.get("file") == "weights.pt"):
        raise ValueError("Shared weights metadata is required; re-export both packages")
    if path.stat().st_size != contract.get("bytes") or _sha256(path) != contract.get("sha256"):
        raise ValueError("Shared weights archive checksum mismatch")
    if read_manifest(path)["identity_sha256"] != contract.get("identity"):
        raise ValueError("Shared weights identity mismatch")


def load_weights(directory, device="cpu", verify=True):
    """{HF name: tensor} of a bundle directory's weights.pt (views over shared storages).

    With verify=True and a decode.json sidecar present, its `shared_weights` contract is checked
    first."""
    directory = Path(directory)
    path = directory / "weights.pt"
    if verify and (directory / "decode.json").is_file():
        meta = json.loads((directory / "decode.json").read_text())
        check_contract(directory, meta.get("shared_weights"))
    data = read_manifest(path)
    archive = torch.jit.load(str(path), map_location="cpu")
    if getattr(archive, "identity", None) != data["identity_sha256"]:
        raise ValueError("Shared weights archive identity mismatch")
    storages = dict(archive.named_buffers())
    if set(storages) != set(data["storages"]):
        raise ValueError("Shared weights archive buffer set mismatch")
    moved = {}
    for name, t in storages.items():
        d = data["storages"][name]
        if (t.ndim != 1 or str(t.dtype).removeprefix("torch.") != d["dtype"]
                or t.numel() * t.element_size() != d["bytes"]):
            raise ValueError("Shared weights archive tensor metadata mismatch")
        moved[name] = t.to(device)
    out = {}
    for exported, view in data["sources"].items():
        d = data["tensors"][view]
        base = moved[d["storage"]]
        out[hf_name(exported)] = base.as_strided(d["shape"], d["stride"], d["offset"])
    return out


def engine_weights(geometry, weights):
    """The subset of `weights` the Engine takes, checked against the geometry's HF shapes."""
    out = {}
    for name, (shape, _) in synthetic.parameter_shapes(geometry).items():
        if name not in weights:
            raise ValueError(f"bundle lacks {name}")
        t = weights[name]
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: bundle shape {tuple(t.shape)} != {tuple(shape)}")
        out[name] = t.contiguous() if t.dtype == torch.bfloat16 else t.to(torch.bfloat16).contiguous()
    out["lm_head.weight"] = weights.get("lm_head.weight", out["model.embed_tokens.weight"])
    if out["lm_head.weight"].data_ptr() != out["model.embed_tokens.weight"].data_ptr():
        out["lm_head.weight"] = out["lm_head.weight"].contiguous()
    return out
