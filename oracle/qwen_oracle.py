"""CPU ORACLE for the Qwen2 decode path — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` use it, and only as the checker or as the
timed CPU baseline, never as a code path of the engine.

It restates, in fp32 PyTorch on the CPU, the math of SeedPlane's portable decoder
`seedplane/qwen_engine.py` (the reference every SeedPlane backend must match token for token,
`qwen_engine.py:5-7`):

* `OracleQwen2.__init__`  -- QKV / gate-up fusion, fp32 norm gains   (qwen_engine.py:64-80)
* `OracleQwen2.norm`      -- RMSNorm x * rsqrt(mean(x^2) + eps) * g (qwen_engine.py:90-92)
* `OracleQwen2.rope`      -- fp32 inv_freq and phase, rotate-half    (qwen_engine.py:52,94-103)
* `OracleQwen2.forward`   -- embed, L x {norm, QKV+bias, RoPE, cache write, GQA attention with
                             the slot mask, O + residual, norm, gate/up, SiLU*up, down + residual},
                             final norm, LM head on the last row or all rows (qwen_engine.py:105-144)
* `OracleQwen2.greedy`    -- greedy generate loop, argmax = first index of the max
                             (qwen_engine.py:147-148,158-166)

Two options the reference lacks but the B200 engine needs a checker for:

* `kv_fp16=True` rounds K and V to fp16 when they are written to the cache (the engine keeps an
  fp16 KV cache; the reference does this only implicitly on GPU where it computes in fp16).
* `forward(..., visible=mask)` replaces the slot mask by an explicit [q, start+q] boolean mask,
  which is how tree verification (each node sees the committed prefix and its ancestors) is
  checked. With `visible=None` the mask is the reference's `arange <= slot`.

Weights may be given as fp16 / fp32 tensors, or as blockwise int8 (`<name>` int8 plus
`<name>.scales` fp16, 32-element blocks), which is dequantized exactly to fp32.

Pinned against: golden tokens and logits produced by running the reference `Qwen2Engine` itself
(`tests/golden/make_golden.py`), checked in `tests/test_oracle_golden.py`.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.nn.functional as F


@dataclass
class OracleCache:
    """Per-layer K/V of shape [capacity, kv_heads, head_dim] in fp32 (`qwen_engine.py:18-29`)."""
    keys: list
    values: list
    length: int
    capacity: int

    def clone(self) -> "OracleCache":
        return OracleCache([k.clone() for k in self.keys], [v.clone() for v in self.values],
                           self.length, self.capacity)


def _dequant(q: torch.Tensor, s: torch.Tensor, block: int = 32) -> torch.Tensor:
    n, k = q.shape
    return (q.float().view(n, k // block, block) * s.float().view(n, k // block, 1)).view(n, k)


class OracleQwen2:
    def __init__(self, cfg, weights: Dict[str, torch.Tensor], kv_fp16: bool = False, layers: Optional[int] = None):
        self.cfg = cfg
        self.L = cfg.layers if layers is None else layers
        self.H, self.NH, self.NKV, self.HD = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        self.eps = cfg.rms_norm_eps
        self.kv_fp16 = kv_fp16

        def get(name):
            t = weights[name]
            if t.dtype == torch.int8:
                return _dequant(t, weights[name + ".scales"])
            return t.float()

        self.embed = get("model.embed_tokens.weight")
        self.head = get("lm_head.weight") if "lm_head.weight" in weights else self.embed
        self.final_norm = get("model.norm.weight")
        self.layers = []
        for l in range(self.L):
            p = f"model.layers.{l}."
            self.layers.append({
                "qkv_w": torch.cat([get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"),
                                    get(p + "self_attn.v_proj.weight")]),
                "qkv_b": torch.cat([get(p + "self_attn.q_proj.bias"), get(p + "self_attn.k_proj.bias"),
                                    get(p + "self_attn.v_proj.bias")]),
                "o_w": get(p + "self_attn.o_proj.weight"),
                "gate_up_w": torch.cat([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")]),
                "down_w": get(p + "mlp.down_proj.weight"),
                "in_norm": get(p + "input_layernorm.weight"),
                "post_norm": get(p + "post_attention_layernorm.weight"),
            })
        half = torch.arange(0, self.HD, 2).float() / self.HD
        self.inv_freq = 1.0 / (float(cfg.rope_theta) ** half)

    # -- pieces -----------------------------------------------------------------------------
    def new_cache(self, capacity: int) -> OracleCache:
        capacity = min(capacity, self.cfg.max_positions)
        if capacity < 1:
            raise ValueError("cache capacity must be positive")
        shape = (capacity, self.NKV, self.HD)
        return OracleCache([torch.zeros(shape) for _ in range(self.L)],
                           [torch.zeros(shape) for _ in range(self.L)], 0, capacity)

    def norm(self, x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * g

    def rope_table(self, positions: torch.Tensor):
        """cos/sin [q, HD] in fp32, the phase duplicated over both halves of a head."""
        phase = positions.float()[:, None] * self.inv_freq[None, :]
        phase = torch.cat([phase, phase], dim=-1)
        return phase.cos(), phase.sin()

    @staticmethod
    def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """x [q, heads, HD]; rotate-half pairs (i, i + HD/2)."""
        h = x.shape[-1] // 2
        rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
        return x * cos[:, None, :] + rot * sin[:, None, :]

    # -- forward ----------------------------------------------------------------------------
    @torch.inference_mode()
    def forward(self, ids: Sequence[int], cache: Optional[OracleCache] = None, all_logits: bool = False,
                positions: Optional[Sequence[int]] = None, visible: Optional[torch.Tensor] = None,
                slots: Optional[Sequence[int]] = None, advance: bool = True):
        """Logits (fp32 [q or 1, V]) and the cache, like `Qwen2Engine.forward`.

        `slots` (default start..start+q) are the cache rows written; `visible` [q, n_keys] is an
        explicit attention mask over cache rows 0..n_keys-1 (default: rows <= own slot).
        `advance=False` leaves `cache.length` untouched (speculative nodes are scratch rows).
        """
        ids_t = torch.as_tensor(list(ids), dtype=torch.long).flatten()
        q = ids_t.numel()
        if q == 0:
            raise ValueError("input_ids cannot be empty")
        if cache is None:
            cache = self.new_cache(4096)
        start = cache.length
        slot_t = torch.arange(start, start + q) if slots is None else torch.as_tensor(list(slots), dtype=torch.long)
        if int(slot_t.max()) >= cache.capacity:
            raise ValueError(f"KV cache capacity {cache.capacity} exceeded")
        pos_t = slot_t if positions is None else torch.as_tensor(list(positions), dtype=torch.long).flatten()
        if pos_t.numel() != q:
            raise ValueError("positions must match input_ids")
        n_keys = int(slot_t.max()) + 1 if visible is None else visible.shape[1]
        if visible is None:
            visible = torch.arange(n_keys)[None, :] <= slot_t[:, None]
        cos, sin = self.rope_table(pos_t)
        scale = 1.0 / (self.HD ** 0.5)
        G = self.NH // self.NKV

        x = self.embed[ids_t]
        for l in range(self.L):
            ly = self.layers[l]
            h = self.norm(x, ly["in_norm"])
            qkv = h @ ly["qkv_w"].T + ly["qkv_b"]
            qh = qkv[:, :self.NH * self.HD].view(q, self.NH, self.HD)
            kh = qkv[:, self.NH * self.HD:(self.NH + self.NKV) * self.HD].view(q, self.NKV, self.HD)
            vh = qkv[:, (self.NH + self.NKV) * self.HD:].view(q, self.NKV, self.HD)
            qh, kh = self.rope(qh, cos, sin), self.rope(kh, cos, sin)
            if self.kv_fp16:
                kh, vh = kh.half().float(), vh.half().float()
            cache.keys[l][slot_t] = kh
            cache.values[l][slot_t] = vh
            K = cache.keys[l][:n_keys]          # [n, NKV, HD]
            Vv = cache.values[l][:n_keys]
            out = torch.empty(q, self.NH, self.HD)
            for g in range(self.NKV):
                qg = qh[:, g * G:(g + 1) * G, :]                       # [q, G, HD]
                s = torch.einsum("qgd,nd->qgn", qg, K[:, g, :]) * scale
                s = s.masked_fill(~visible[:, None, :], float("-inf"))
                p = torch.softmax(s, dim=-1)
                out[:, g * G:(g + 1) * G, :] = torch.einsum("qgn,nd->qgd", p, Vv[:, g, :])
            x = x + out.reshape(q, self.H) @ ly["o_w"].T
            h = self.norm(x, ly["post_norm"])
            gu = h @ ly["gate_up_w"].T
            gate, up = gu[:, :self.cfg.intermediate], gu[:, self.cfg.intermediate:]
            x = x + (F.silu(gate) * up) @ ly["down_w"].T
        if advance:
            cache.length = max(cache.length, int(slot_t.max()) + 1)
        xf = self.norm(x if all_logits else x[-1:], self.final_norm)
        return xf @ self.head.T, cache

    @torch.inference_mode()
    def greedy(self, prompt: Sequence[int], n_new: int, capacity: Optional[int] = None):
        """Greedy tokens plus the top-1/top-2 logit margin of each step (`qwen_engine.py:158-166`)."""
        cache = self.new_cache(capacity or len(prompt) + n_new)
        logits, cache = self.forward(prompt, cache)
        tokens: List[int] = []
        margins: List[float] = []
        for i in range(n_new):
            row = logits[-1]
            top = torch.topk(row, 2)
            tokens.append(int(row.argmax()))
            margins.append(float(top.values[0] - top.values[1]))
            if i + 1 < n_new:
                logits, cache = self.forward([tokens[-1]], cache)
        return tokens, margins

    @torch.inference_mode()
    def prefix_logits(self, tokens: Sequence[int]) -> torch.Tensor:
        """Logits for the next token after `tokens`, computed from an empty cache."""
        logits, _ = self.forward(tokens, self.new_cache(len(tokens)))
        return logits[-1]
