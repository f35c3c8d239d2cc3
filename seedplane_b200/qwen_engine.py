"""Drop-in for SeedPlane's `seedplane.qwen_engine` backed by the B200 CUDA engine.

Same surface as the reference (`seedplane/qwen_engine.py:18-172`):

* `KVCache` with `length` / `capacity` (the K/V live in the engine's fp16 device cache; setting
  `length` rolls the cache back, as `experiments/hive_scaling/benchmark_speculative.py:119` does),
* `Qwen2Engine(bundle, device, dtype)` with `new_cache`, `forward(input_ids, cache, all_logits,
  positions) -> (fp32 logits [q or 1, V], cache)`, `sample`, `generate`,
* `chat_prompt(messages)`.

Differences that a caller can observe: logits are returned on the CUDA device; weights are held
in fp16 and K/V in fp16 while every activation and accumulation is fp32; `dtype` may only be
None or torch.float16. The engine refuses to run without a CUDA device (no CPU fallback).

Besides HF directories, `bundle` may be a seedplane-bundle/2 directory (`seedplane.json` +
`weights.spw`, `seedplane/native_bundle.py:62-137`), or weights may be passed directly with
`config=` and `weights=` (the random-init checkpoints of the benchmarks).
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Optional

import torch

from .bundle import load_checkpoint
from .config import Qwen2Config
from .engine import CudaQwen2, DeviceKV


class KVCache:
    """Handle of one device KV cache (`qwen_engine.py:18-29`)."""

    def __init__(self, dkv: DeviceKV):
        self.device_kv = dkv

    @property
    def length(self) -> int:
        return self.device_kv.length

    @length.setter
    def length(self, n: int):
        self.device_kv.length = n

    @property
    def capacity(self) -> int:
        return self.device_kv.capacity


class Qwen2Engine:
    """Inference-only Qwen2/Qwen2.5 runtime with a persistent device KV cache."""

    def __init__(self, bundle=None, device="cuda", dtype=None, *, config: Optional[Qwen2Config] = None,
                 weights: Optional[Dict[str, torch.Tensor]] = None, weight_format: str = "f16"):
        if dtype not in (None, torch.float16):
            raise ValueError("the B200 engine holds fp16 weights (fp32 activations); dtype must be None or float16")
        if bundle is not None:
            self.bundle = Path(bundle)
            config, weights, weight_format = load_checkpoint(self.bundle)
        elif config is None or weights is None:
            raise ValueError("give a bundle directory, or config= and weights=")
        else:
            self.bundle = None
        self.cfg = config
        self.config = config.to_hf()
        self.device = torch.device(device)
        self.dtype = torch.float16
        self.n_layers, self.n_heads, self.n_kv_heads = config.layers, config.heads, config.kv_heads
        self.hidden, self.head_dim = config.hidden, config.head_dim
        self.eps = config.rms_norm_eps
        self.engine = CudaQwen2(config, weights, device=self.device, weight_format=weight_format)
        self.device = self.engine.device

    def new_cache(self, capacity=4096) -> KVCache:
        capacity = min(capacity, self.config["max_position_embeddings"])
        if capacity < 1:
            raise ValueError("cache capacity must be positive")
        return KVCache(self.engine.new_kv(capacity))

    @torch.inference_mode()
    def forward(self, input_ids, cache=None, all_logits=False, positions=None):
        """Run tokens through the graph; `positions` (default: cache slots) are the RoPE position ids."""
        ids = torch.as_tensor(input_ids, dtype=torch.long).flatten()
        if ids.numel() == 0:
            raise ValueError("input_ids cannot be empty")
        if cache is None:
            cache = self.new_cache()
        start, qlen = cache.length, ids.numel()
        if start + qlen > cache.capacity:
            raise ValueError(f"KV cache capacity {cache.capacity} exceeded")
        if positions is not None:
            positions = torch.as_tensor(positions, dtype=torch.long).flatten()
            if positions.numel() != qlen:
                raise ValueError("positions must match input_ids")
        logits, _ = self.engine.forward(cache.device_kv, ids.to(torch.int32), positions, all_logits=all_logits)
        return logits, cache

    @staticmethod
    def sample(logits, temperature=0.0, top_k=0, top_p=1.0, generator=None):
        """Greedy argmax (first index of the max) or temperature / top-k / top-p sampling
        (the reference's definition, `qwen_engine.py:146-156`)."""
        if temperature <= 0:
            return int(logits.argmax())
        z = logits / temperature
        if top_k > 0:
            cutoff = torch.topk(z, min(top_k, z.numel())).values[-1]
            z = z.masked_fill(z < cutoff, -torch.inf)
        if top_p < 1:
            values, indices = torch.sort(z, descending=True)
            probs = values.softmax(-1)
            drop = probs.cumsum(-1) - probs > top_p
            values = values.masked_fill(drop, -torch.inf)
            z = torch.full_like(z, -torch.inf).scatter(0, indices, values)
        return int(torch.multinomial(z.softmax(-1), 1, generator=generator))

    @torch.inference_mode()
    def generate(self, prompt_ids, max_new_tokens=128, temperature=0.0, top_k=0, top_p=1.0, eos_token_id=None,
                 seed=1, block=32):
        """Yield generated token ids (`qwen_engine.py:158-166`).

        Greedy decoding runs `block` tokens per device call with the argmax fed back on the GPU
        (no host round trip per token); the token sequence is the same as one-at-a-time.
        """
        cache = self.new_cache(len(prompt_ids) + max_new_tokens)
        if temperature > 0:
            logits, cache = self.forward(prompt_ids, cache)
            gen = torch.Generator(device=self.device).manual_seed(seed)
            for _ in range(max_new_tokens):
                token = self.sample(logits[-1], temperature, top_k, top_p, gen)
                yield token
                if token == eos_token_id:
                    break
                logits, cache = self.forward([token], cache)
            return
        _, argmax = self.engine.forward(cache.device_kv, torch.as_tensor(list(prompt_ids), dtype=torch.int32),
                                        want_logits=False)
        token = int(argmax[-1])
        yield token
        produced = 1
        if token == eos_token_id:
            return
        pos = cache.length
        while produced < max_new_tokens:
            n = min(block, max_new_tokens - produced)
            out, _ = self.engine.decode(cache.device_kv, token, pos, n)
            toks = out.tolist()
            for t in toks:
                yield t
                produced += 1
                if t == eos_token_id:
                    return
            token = toks[-1]
            pos += n


def chat_prompt(messages):
    """Render Qwen's ChatML without depending on Transformers (`qwen_engine.py:169-172`)."""
    text = "".join(f"<|im_start|>{m['role']}\n{m['content']}<|im_end|>\n" for m in messages)
    return text + "<|im_start|>assistant\n"
