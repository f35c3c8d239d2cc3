"""Checkpoint loading for the B200 engine.

Two on-disk formats are accepted:

* an HF directory (`config.json` + `*.safetensors`), what `Qwen2Engine` loads
  (`seedplane/qwen_engine.py:35-63`);
* a seedplane-bundle/2 directory (`seedplane.json` + `weights.spw`), what the native runtime loads
  (`seedplane/native_bundle.py:62-137`, `native/vulkan_decode/qwen_vk.cpp:63-85`): a JSON manifest
  with an `arch` block and a tensor table of {dtype f16|f32, shape, offset, bytes} into one
  256-byte-aligned blob, tensors `embed`, `lm_head` (untied only), `final_norm`, `{l}.qkv_w`,
  `{l}.qkv_b`, `{l}.o_w`, `{l}.gate_w`, `{l}.up_w`, `{l}.down_w`, `{l}.in_norm`, `{l}.post_norm`.

Int8 blockwise checkpoints (this engine's extension) store `<name>` int8 and `<name>.scales`
fp16 side by side in safetensors.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from .config import Qwen2Config

BUNDLE_FORMAT = "seedplane-bundle/2"


def load_checkpoint(path) -> Tuple[Qwen2Config, Dict[str, torch.Tensor], str]:
    """(config, tensors, weight_format) from an HF directory or a seedplane-bundle/2 directory."""
    p = Path(path)
    if (p / "seedplane.json").exists() and (p / "weights.spw").exists():
        meta = json.loads((p / "seedplane.json").read_text())
        if meta.get("format") == BUNDLE_FORMAT:
            return load_bundle_v2(p)
    if not (p / "config.json").exists():
        raise FileNotFoundError(f"{p}: neither an HF checkpoint directory nor a {BUNDLE_FORMAT} bundle")
    cfg = Qwen2Config.from_hf(json.loads((p / "config.json").read_text()), name=p.name)
    files = sorted(p.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors in {p}")
    from safetensors import safe_open
    w: Dict[str, torch.Tensor] = {}
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as fh:
            for name in fh.keys():
                if name in w:
                    raise ValueError(f"duplicate tensor {name}")
                w[name] = fh.get_tensor(name)
    required = {"model.embed_tokens.weight", "model.norm.weight"}
    if not required.issubset(w):
        raise ValueError("bundle is missing Qwen2 tensors")
    if "lm_head.weight" in w and cfg.tied_embeddings:
        from dataclasses import replace
        cfg = replace(cfg, tied_embeddings=False)
    fmt = "i8" if w.get("model.layers.0.self_attn.q_proj.weight", torch.empty(0)).dtype == torch.int8 else "f16"
    return cfg, w, fmt


def load_bundle_v2(path, verify_sha256: bool = False) -> Tuple[Qwen2Config, Dict[str, torch.Tensor], str]:
    p = Path(path)
    meta = json.loads((p / "seedplane.json").read_text())
    if meta.get("format") != BUNDLE_FORMAT:
        raise ValueError(f"{p}: not a {BUNDLE_FORMAT} bundle")
    cfg = Qwen2Config.from_bundle_arch(meta["arch"], name=p.name)
    blob = np.memmap(p / "weights.spw", dtype=np.uint8, mode="r")
    if verify_sha256:
        digest = hashlib.sha256(blob.tobytes()).hexdigest()
        if digest != meta["weights"]["sha256"]:
            raise ValueError(f"{p}: weights.spw sha256 mismatch")
    out: Dict[str, torch.Tensor] = {}
    for name, t in meta["tensors"].items():
        raw = blob[t["offset"]:t["offset"] + t["bytes"]]
        dt = {"f16": "<f2", "f32": "<f4"}[t["dtype"]]
        out[name] = torch.from_numpy(np.array(raw.view(dt)).reshape(t["shape"]))
    return cfg, out, "f16"


def bundle_plan(path) -> Optional[dict]:
    """The shard plan a SeedPlane bundle carries (`seedplane.json` `plan`), or None."""
    p = Path(path)
    if (p / "seedplane.json").exists():
        meta = json.loads((p / "seedplane.json").read_text())
        if "plan" in meta:
            return dict(meta["plan"])
    return None


def plan_of(path) -> dict:
    """The shard plan of a bundle (`seedplane.json` `plan`), or the reference default."""
    plan = bundle_plan(path)
    return plan if plan is not None else {"shard": 512, "halo": 256, "sinks": 4}
