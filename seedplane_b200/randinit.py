"""Seeded random-init Qwen2 checkpoints (the synthetic stand-in for real weights).

Every benchmark configuration is a random-init model: weights, embeddings and biases are drawn
from N(0, std) with `torch.Generator().manual_seed(seed)` on the CPU, RMSNorm gains are 1.
Tensors are drawn one after another in this fixed order (HF names):

    model.embed_tokens.weight
    for each layer l:  q_proj.weight, q_proj.bias, k_proj.weight, k_proj.bias, v_proj.weight,
                       v_proj.bias, o_proj.weight, gate_proj.weight, up_proj.weight, down_proj.weight
    lm_head.weight     (untied models only)

`dtype=torch.float16` rounds each tensor to fp16 round-to-nearest-even right after drawing it,
which is what SeedPlane's bundle converter does to matrices (`seedplane/native_bundle.py:93-98`).
The fp16-rounded checkpoint is the one both the CUDA engine and the CPU oracle run.

The int8 variant (`make_int8_blockwise`) draws, per matrix, int8 values uniform in [-127, 127]
and one fp16 scale per 32-element block along the input dimension with scale = |N(0, std)|/127.
"""
from __future__ import annotations

import hashlib
from typing import Dict, Iterator, Tuple

import torch

from .config import Qwen2Config

# Init used by the tiny parity-test models (N(0, 0.02) makes tiny tied models repeat one token).
TEST_INIT = {"std": 0.1, "embed_std": 0.5}

LAYER_TENSORS = ("self_attn.q_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.weight",
                 "self_attn.k_proj.bias", "self_attn.v_proj.weight", "self_attn.v_proj.bias",
                 "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                 "mlp.down_proj.weight")
MATRIX_SUFFIXES = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                   "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                   "mlp.down_proj.weight")


def tensor_shapes(cfg: Qwen2Config) -> Iterator[Tuple[str, tuple]]:
    """Drawn tensors in generation order, with their HF shapes."""
    H, NH, NKV, HD, I, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab
    shapes = {"self_attn.q_proj.weight": (NH * HD, H), "self_attn.q_proj.bias": (NH * HD,),
              "self_attn.k_proj.weight": (NKV * HD, H), "self_attn.k_proj.bias": (NKV * HD,),
              "self_attn.v_proj.weight": (NKV * HD, H), "self_attn.v_proj.bias": (NKV * HD,),
              "self_attn.o_proj.weight": (H, H), "mlp.gate_proj.weight": (I, H),
              "mlp.up_proj.weight": (I, H), "mlp.down_proj.weight": (H, I)}
    yield "model.embed_tokens.weight", (V, H)
    for layer in range(cfg.layers):
        for suffix in LAYER_TENSORS:
            yield f"model.layers.{layer}.{suffix}", shapes[suffix]
    if not cfg.tied_embeddings:
        yield "lm_head.weight", (V, H)


def make_weights(cfg: Qwen2Config, seed: int = 0, std: float = 0.02,
                 dtype: torch.dtype = torch.float16, embed_std: float = None) -> Dict[str, torch.Tensor]:
    """HF-named CPU tensors of a seeded random-init Qwen2 checkpoint (norm gains = 1).

    `embed_std` (default `std`) is the spread of the embedding matrix alone; the tiny test
    models use std 0.1 / embed_std 0.5 so that greedy output is diverse (TEST_INIT).
    """
    g = torch.Generator().manual_seed(seed)
    w: Dict[str, torch.Tensor] = {}
    for name, shape in tensor_shapes(cfg):
        s = embed_std if (embed_std is not None and name == "model.embed_tokens.weight") else std
        t = torch.empty(shape, dtype=torch.float32).normal_(0.0, s, generator=g)
        w[name] = t.to(dtype) if dtype != torch.float32 else t
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}."
        w[p + "input_layernorm.weight"] = torch.ones(cfg.hidden, dtype=dtype)
        w[p + "post_attention_layernorm.weight"] = torch.ones(cfg.hidden, dtype=dtype)
    w["model.norm.weight"] = torch.ones(cfg.hidden, dtype=dtype)
    return w


def make_int8_blockwise(cfg: Qwen2Config, seed: int = 0, std: float = 0.02, block: int = 32,
                        device: str = "cpu") -> Dict[str, torch.Tensor]:
    """Blockwise-int8 checkpoint: `<name>` int8 [N, K] and `<name>.scales` fp16 [N, K/block].

    Matrices of every layer (and an untied LM head) are int8; the embedding, biases and norm
    gains stay fp16 / fp32. Values: int8 uniform in [-127, 127], scale = |N(0, std)| / 127.
    `device="cuda"` draws on the GPU with a CUDA generator (different values from the CPU
    stream for the same seed; used only where no CPU oracle needs the same tensors).
    """
    g = torch.Generator(device=device).manual_seed(seed)
    w: Dict[str, torch.Tensor] = {}
    for name, shape in tensor_shapes(cfg):
        is_matrix = name == "lm_head.weight" or any(name.endswith(s) for s in MATRIX_SUFFIXES)
        if is_matrix:
            n, k = shape
            if k % block:
                raise ValueError(f"{name}: K={k} is not a multiple of the {block}-element block")
            w[name] = torch.randint(-127, 128, shape, generator=g, dtype=torch.int8, device=device)
            s = torch.empty((n, k // block), dtype=torch.float32, device=device).normal_(0.0, std, generator=g)
            w[name + ".scales"] = (s.abs() / 127.0).to(torch.float16)
        else:
            w[name] = torch.empty(shape, dtype=torch.float32, device=device).normal_(
                0.0, std, generator=g).to(torch.float16)
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}."
        w[p + "input_layernorm.weight"] = torch.ones(cfg.hidden, dtype=torch.float16, device=device)
        w[p + "post_attention_layernorm.weight"] = torch.ones(cfg.hidden, dtype=torch.float16, device=device)
    w["model.norm.weight"] = torch.ones(cfg.hidden, dtype=torch.float16, device=device)
    return w


def dequantize_int8(q: torch.Tensor, scales: torch.Tensor, block: int = 32) -> torch.Tensor:
    """fp32 weights w[n, k] = q[n, k] * scale[n, k // block] (exact in fp32: 8 x 11 mantissa bits)."""
    n, k = q.shape
    return (q.float().view(n, k // block, block) * scales.float().view(n, k // block, 1)).view(n, k)


def truncate(weights: Dict[str, torch.Tensor], cfg: Qwen2Config, layers: int) -> Dict[str, torch.Tensor]:
    """The first `layers` layers + final norm + LM head of a checkpoint (the drafter of the verify configs)."""
    keep = {}
    for name, t in weights.items():
        if name.startswith("model.layers."):
            if int(name.split(".")[2]) < layers:
                keep[name] = t
        else:
            keep[name] = t
    return keep


def checksum(weights: Dict[str, torch.Tensor]) -> str:
    """sha256 over the raw bytes of every tensor in sorted-name order (identifies a checkpoint)."""
    h = hashlib.sha256()
    for name in sorted(weights):
        t = weights[name].detach().cpu().contiguous()
        h.update(name.encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else t.numpy().tobytes())
    return h.hexdigest()


def random_prompt(vocab: int, length: int, seed: int = 0) -> list:
    """Uniform-random prompt token ids (`torch.randint(0, V, (P,), generator=manual_seed(seed))`)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (length,), generator=g).tolist()


def burst_prompts(vocab: int, count: int = 16, low: int = 32, high: int = 128, seed: int = 0) -> list:
    """The independent-request burst: `count` prompts, lengths uniform in [low, high], random ids.

    Lengths come from a second generator seeded `seed + 1`; request i's ids from seed `seed + 100 + i`.
    """
    g = torch.Generator().manual_seed(seed + 1)
    lengths = torch.randint(low, high + 1, (count,), generator=g).tolist()
    return [random_prompt(vocab, n, seed + 100 + i) for i, n in enumerate(lengths)]
