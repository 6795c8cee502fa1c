"""Model bundles: the released HS-Guard directory layout, verified and loaded without transformers or safetensors.

A bundle directory holds ``hs_guard.json`` (manifest: ``format`` = ``hs-guard-v1``, ``risk_labels`` = (safe, unsafe,
controversial), ``files`` = {relative path: sha256}, plus ``thresholds`` per head and ``window_tokens``),
``config.json`` (the backbone's transformers config), ``tokenizer.json`` and ``model.safetensors`` (the reference
``Classifier`` state dict: ``backbone.*`` and ``heads.{user,assistant}.*``).

- ``verify_bundle`` applies the reference's manifest rules (src/hs_guard/runtime.py:19-41): known format and label
  order, the three required assets, no absolute or ``..`` paths, every asset a regular file inside the bundle -- or,
  for a hub snapshot (``.../snapshots/<rev>/``), inside the repository's ``blobs`` cache -- and matching its sha256.
- ``read_safetensors`` reads the public safetensors layout (little-endian u64 header size, JSON header of
  {name: {dtype, shape, data_offsets}}, raw little-endian data) into torch tensors.
- ``load_bundle`` returns (model, metadata) for ``StreamingGuard`` / ``SlotEngine``: the model carries the config and
  state dict; ``head='general'`` selects the general heads (the swap of runtime.py:120-122, done by
  ``weights.extract_state_dict``); metadata gets ``head`` and that head's ``thresholds`` as in runtime.py:125.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from .config import HsgConfig, LABELS

FORMAT = "hs-guard-v1"
REQUIRED = ("config.json", "tokenizer.json", "model.safetensors")
_DTYPES = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, None), "F32": (np.float32, None),
           "F64": (np.float64, None), "I64": (np.int64, None), "I32": (np.int32, None), "I16": (np.int16, None),
           "I8": (np.int8, None), "U8": (np.uint8, None), "BOOL": (np.bool_, None)}


def file_sha256(path, block=8 << 20):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            chunk = f.read(block)
            if not chunk:
                return h.hexdigest()
            h.update(chunk)


def _allowed_location(resolved: Path, root: Path) -> bool:
    if resolved.is_relative_to(root):
        return True
    # hub snapshots link immutable assets into <repo>/blobs
    return root.parent.name == "snapshots" and resolved.is_relative_to((root.parent.parent / "blobs").resolve())


def verify_bundle(directory):
    """The bundle's manifest after checking every listed asset; ValueError on any violation."""
    root = Path(directory).resolve()
    manifest = json.loads((root / "hs_guard.json").read_text())
    if manifest.get("format") != FORMAT or manifest.get("risk_labels") != list(LABELS):
        raise ValueError("Unsupported model format or risk-label order")
    files = manifest.get("files", {})
    if not all(name in files for name in REQUIRED):
        raise ValueError("Model manifest is missing required assets")
    for name, digest in files.items():
        rel = Path(name)
        if rel.is_absolute() or ".." in rel.parts:
            raise ValueError(f"Invalid model asset: {name}")
        path = root / rel
        if not path.is_file() or not _allowed_location(path.resolve(), root):
            raise ValueError(f"Invalid model asset: {name}")
        if file_sha256(path) != digest:
            raise ValueError(f"Model asset checksum mismatch: {name}")
    return manifest


def read_safetensors(path):
    """{name: tensor} from a .safetensors file (CPU tensors; bf16 kept as bf16)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError("truncated safetensors header")
        (n,) = struct.unpack("<Q", raw)
        header = json.loads(f.read(n))
    base = 8 + n
    size = os.path.getsize(path)
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=base, shape=(size - base,)) if size > base else None
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in _DTYPES:
            raise ValueError(f"unsupported safetensors dtype {info['dtype']} for {name}")
        np_dtype, torch_view = _DTYPES[info["dtype"]]
        begin, end = info["data_offsets"]
        count = int(np.prod(info["shape"], dtype=np.int64))
        if end - begin != count * np.dtype(np_dtype).itemsize or end > size - base:
            raise ValueError(f"inconsistent data offsets for {name}")
        arr = np.frombuffer(data, dtype=np_dtype, count=count, offset=begin).reshape(info["shape"]).copy() \
            if count else np.zeros(info["shape"], dtype=np_dtype)
        t = torch.from_numpy(arr.view(np.int16) if torch_view is not None else arr)
        out[name] = t.view(torch_view) if torch_view is not None else t
    return out


def config_from_json(cfg_json, window=512):
    """HsgConfig from a transformers Qwen3_5 text config dict (nested ``text_config`` accepted)."""
    d = dict(cfg_json.get("text_config", cfg_json))
    if "layer_types" not in d:
        interval = d.get("full_attention_interval", 4)
        d["layer_types"] = ["full_attention" if (i + 1) % interval == 0 else "linear_attention"
                            for i in range(d["num_hidden_layers"])]
    if "rope_parameters" not in d:
        d["rope_parameters"] = {"rope_theta": d.get("rope_theta", 10000.0),
                                "partial_rotary_factor": d.get("partial_rotary_factor", 0.25)}
    return HsgConfig.from_hf(SimpleNamespace(**d), window=window)


class BundleModel:
    """A loaded bundle as the engine consumes it: ``cfg`` and ``state_dict()`` (reference parameter names)."""

    def __init__(self, cfg, state_dict):
        self.cfg, self._sd = cfg, state_dict

    def state_dict(self):
        return self._sd


def load_bundle(directory, head="redline"):
    """(BundleModel, metadata) of a verified bundle directory (reference runtime.py:97-126 without the hub
    download: pass a local snapshot directory)."""
    if head not in ("redline", "general"):
        raise ValueError("head must be redline or general")
    root = Path(directory)
    manifest = verify_bundle(root)
    window = int(manifest.get("window_tokens", 512))
    cfg = config_from_json(json.loads((root / "config.json").read_text()), window=window)
    sd = read_safetensors(root / "model.safetensors")
    metadata = dict(manifest, head=head)
    if isinstance(manifest.get("thresholds"), dict) and head in manifest["thresholds"]:
        metadata["thresholds"] = manifest["thresholds"][head]
    return BundleModel(cfg, sd), metadata
