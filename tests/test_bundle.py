"""Bundle verification and loading (hs_guard_b200.bundle): the reference's manifest rules (its
tests/test_contract.py ManifestTests cases, restated), the safetensors reader, config parsing and head selection."""
import hashlib
import json
import struct

import numpy as np
import pytest
import torch

from hs_guard_b200 import DEFAULT
from hs_guard_b200.bundle import config_from_json, load_bundle, read_safetensors, verify_bundle
from hs_guard_b200.weights import extract_state_dict

_CODES = {torch.bfloat16: "BF16", torch.float32: "F32", torch.int64: "I64", torch.float16: "F16"}


def write_safetensors(path, tensors):
    """Test-side writer of the safetensors layout (header size, JSON header, raw little-endian data)."""
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        raw = t.contiguous().view(torch.int16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
        header[name] = {"dtype": _CODES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def _digest(path):
    return hashlib.sha256(path.read_bytes()).hexdigest()


def _bundle(root, tensors, extra_manifest=None):
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(json.dumps(DEFAULT.hf_kwargs()))
    (root / "tokenizer.json").write_text("{}")
    write_safetensors(root / "model.safetensors", tensors)
    files = {n: _digest(root / n) for n in ("config.json", "tokenizer.json", "model.safetensors")}
    manifest = {"format": "hs-guard-v1", "risk_labels": ["safe", "unsafe", "controversial"], "files": files,
                "window_tokens": 512,
                "thresholds": {"redline": {"user": 0.07, "assistant": 0.11}, "general": {"user": 0.5, "assistant": 0.6}}}
    manifest.update(extra_manifest or {})
    (root / "hs_guard.json").write_text(json.dumps(manifest))
    return manifest


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    tensors = {"a": torch.randn(3, 5, generator=g).bfloat16(), "b": torch.randn(7, generator=g),
               "c": torch.arange(6, dtype=torch.int64).reshape(2, 3), "d": torch.zeros(0, 4), "e": torch.ones(2).half()}
    write_safetensors(tmp_path / "m.safetensors", tensors)
    back = read_safetensors(tmp_path / "m.safetensors")
    assert set(back) == set(tensors)
    for k, t in tensors.items():
        assert back[k].dtype == t.dtype and back[k].shape == t.shape and torch.equal(back[k], t)


def test_config_json_round_trip():
    assert config_from_json(DEFAULT.hf_kwargs()) == DEFAULT
    assert config_from_json({"text_config": DEFAULT.hf_kwargs()}) == DEFAULT


def test_load_bundle_and_head_selection(tmp_path):
    heads = {}
    for role in ("user", "assistant"):
        for part, shape in (("projection.0.weight", (4, 2)), ("projection.0.bias", (4,)), ("projection.1.weight", (4,)),
                            ("projection.1.bias", (4,)), ("risk.weight", (3, 4)), ("risk.bias", (3,))):
            heads[f"heads.{role}.{part}"] = torch.full(shape, 1.0)
            gpart = part.replace("projection", "general_projection").replace("risk", "general")
            heads[f"heads.{role}.{gpart}"] = torch.full(shape, 2.0)
    _bundle(tmp_path / "b", heads)
    model, meta = load_bundle(tmp_path / "b", head="general")
    assert model.cfg == DEFAULT and meta["head"] == "general" and meta["thresholds"] == {"user": 0.5, "assistant": 0.6}
    cfg, sd = extract_state_dict(model, head="general")
    assert cfg == DEFAULT and torch.equal(sd["heads.user.risk.weight"], torch.full((3, 4), 2.0))
    _, sd = extract_state_dict(model, head="redline")
    assert torch.equal(sd["heads.user.risk.weight"], torch.full((3, 4), 1.0))
    with pytest.raises(ValueError):
        load_bundle(tmp_path / "b", head="other")


def test_hub_snapshot_links_accepted(tmp_path):
    """Assets symlinked from a hub snapshot into the repository's blob cache are accepted."""
    base = tmp_path / "repo"
    root, blobs = base / "snapshots" / "revision", base / "blobs"
    root.mkdir(parents=True)
    blobs.mkdir()
    files = {}
    for name in ("config.json", "tokenizer.json", "model.safetensors"):
        content = name.encode()
        digest = hashlib.sha256(content).hexdigest()
        (blobs / digest).write_bytes(content)
        (root / name).symlink_to("../../blobs/" + digest)
        files[name] = digest
    manifest = {"format": "hs-guard-v1", "risk_labels": ["safe", "unsafe", "controversial"], "files": files}
    (root / "hs_guard.json").write_text(json.dumps(manifest))
    assert verify_bundle(root)["files"] == files
    manifest["files"]["../escape"] = "0" * 64
    (root / "hs_guard.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError):
        verify_bundle(root)


def test_external_symlink_and_bad_manifests_rejected(tmp_path):
    base = tmp_path
    root = base / "bundle"
    root.mkdir()
    files = {}
    for name in ("config.json", "tokenizer.json", "model.safetensors"):
        (base / name).write_text(name)
        (root / name).symlink_to(base / name)
        files[name] = hashlib.sha256(name.encode()).hexdigest()
    (root / "hs_guard.json").write_text(json.dumps(
        {"format": "hs-guard-v1", "risk_labels": ["safe", "unsafe", "controversial"], "files": files}))
    with pytest.raises(ValueError):
        verify_bundle(root)
    good = tmp_path / "good"
    m = _bundle(good, {"x": torch.zeros(2)})
    assert verify_bundle(good)["format"] == "hs-guard-v1"
    for bad in ({"format": "other"}, {"risk_labels": ["unsafe", "safe", "controversial"]},
                {"files": {k: v for k, v in m["files"].items() if k != "tokenizer.json"}},
                {"files": dict(m["files"], **{"config.json": "0" * 64})}, {"files": dict(m["files"], **{"/abs": "0"})}):
        _bundle(good, {"x": torch.zeros(2)}, bad)
        with pytest.raises(ValueError):
            verify_bundle(good)
