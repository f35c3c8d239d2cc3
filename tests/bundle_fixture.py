"""Rebuild a seedplane-bundle/2 directory from a recorded converter manifest (test helper).

`tests/golden/bundle_<name>.json` is the `seedplane.json` that the reference's converter
(`seedplane/native_bundle.py:62-137`) wrote for a seeded random-init checkpoint. The weights blob
is rebuilt here from the same seeded weights by the manifest's tensor table (fused QKV, fp16
matrices, fp32 norms and biases, zero padding to each recorded offset) and must hash to the SHA-256
the converter recorded, so the bundle a test loads is byte-identical to the converter's output.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def manifest(name: str) -> dict:
    return json.loads((GOLDEN / f"bundle_{name}.json").read_text())


def source_tensor(w, cfg, key: str) -> torch.Tensor:
    """The converter's tensor `key` from HF-named weights (same fusion and order)."""
    if key == "embed":
        return w["model.embed_tokens.weight"]
    if key == "lm_head":
        return w["lm_head.weight"]
    if key == "final_norm":
        return w["model.norm.weight"]
    layer, part = key.split(".", 1)
    p = f"model.layers.{int(layer)}."
    if part in ("qkv_w", "qkv_b"):
        kind = "weight" if part == "qkv_w" else "bias"
        return torch.cat([w[p + f"self_attn.{x}_proj.{kind}"] for x in ("q", "k", "v")])
    return w[p + {"o_w": "self_attn.o_proj.weight", "gate_w": "mlp.gate_proj.weight", "up_w": "mlp.up_proj.weight",
                  "down_w": "mlp.down_proj.weight", "in_norm": "input_layernorm.weight",
                  "post_norm": "post_attention_layernorm.weight"}[part]]


def rebuild(name: str, weights, cfg, directory: Path) -> Path:
    """Write `seedplane.json` + `weights.spw` into `directory`; raises if the blob's SHA-256 differs
    from the converter's."""
    meta = manifest(name)
    directory.mkdir(parents=True, exist_ok=True)
    h = hashlib.sha256()
    pos = 0
    with open(directory / "weights.spw", "wb") as f:
        for key, t in sorted(meta["tensors"].items(), key=lambda kv: kv[1]["offset"]):
            if t["offset"] < pos:
                raise ValueError(f"{key}: overlapping tensor table")
            pad = b"\0" * (t["offset"] - pos)
            arr = source_tensor(weights, cfg, key).float().numpy()
            raw = arr.astype("<f2" if t["dtype"] == "f16" else "<f4").tobytes()
            if len(raw) != t["bytes"] or list(arr.shape) != t["shape"]:
                raise ValueError(f"{key}: shape {list(arr.shape)} / {len(raw)} bytes, manifest {t['shape']} / {t['bytes']}")
            for chunk in (pad, raw):
                f.write(chunk)
                h.update(chunk)
            pos = t["offset"] + t["bytes"]
    if h.hexdigest() != meta["weights"]["sha256"]:
        raise ValueError(f"rebuilt weights.spw does not match the converter's sha256 for {name}")
    (directory / "seedplane.json").write_text(json.dumps(meta))
    return directory
