"""CPU ORACLE for shard-window attention — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module; `tests/` use it as the checker of the GPU engine's
windowed sessions (`seedplane_b200/windows.py`).

SeedPlane's defining variant cuts the sequence into shards of S tokens. Position i of shard k
(shard start c0 = k S) attends only to its window: the first `sinks` tokens of the sequence
(fewer when the halo reaches back to them), the H halo tokens before c0, and its own shard up to
itself, all with their ORIGINAL RoPE positions. Two restatements live here:

* `windows` / `visible_indices` / `window_greedy` -- the definition: every position's logits
  recomputed from an empty cache over exactly its window (`seedplane/engine.py:16-33`
  ShardPlan.windows; `experiments/v19/oracle_windows.py:22-33` per-position recomputation).
* `session_greedy` -- the native engine's session, which decodes incrementally into window
  caches and moves between windows at shard boundaries in one of five modes
  (`native/vulkan_decode/qwen_vk.cpp:235,279-301` plan and modes, `:497-570` Session::step,
  `:440-453` copy_slots). The exact modes (rebuild, rebuild-batch, shadow, shadow-batch) give
  the definition's tokens; reuse copies the halo's K/V from the previous window and is an
  approximation, so it has only this restatement as its checker.

The model is `oracle.qwen_oracle.OracleQwen2` (fp32, optional fp16 K/V), its caches written at
explicit slots and positions.
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import torch

MODES = ("full", "rebuild", "rebuild-batch", "shadow", "shadow-batch", "reuse")


def windows(total: int, shard: int, halo: int, sinks: int):
    """(core_start, core_end, visible token indices) per window (`engine.py:27-33`)."""
    if shard <= 0 or halo < 0 or sinks < 0:
        raise ValueError("bad shard plan")
    for c0 in range(0, total, shard):
        c1 = min(total, c0 + shard)
        h0 = max(0, c0 - halo)
        sink = list(range(min(sinks, h0))) if sinks else []
        yield c0, c1, sink + list(range(h0, c1))


def visible_indices(total: int, shard: int, halo: int, sinks: int) -> Dict[int, List[int]]:
    """Position i -> the token indices it reads, ending with i (`oracle_windows.py:25-27`)."""
    vis = {}
    for c0, c1, idx in windows(total, shard, halo, sinks):
        for i in range(c0, c1):
            vis[i] = idx[:len(idx) - (c1 - 1 - i)]
    return vis


@torch.inference_mode()
def window_greedy(model, prompt: Sequence[int], n_new: int, shard: int, halo: int, sinks: int) -> List[int]:
    """Greedy tokens under the window definition: position i's logits from a fresh cache over its
    window with original positions; the argmax after position i >= P - 1 is the next token
    (`oracle_windows.py:28-33`)."""
    seq = [int(t) for t in prompt]
    P, total = len(seq), len(seq) + n_new
    vis = visible_indices(total, shard, halo, sinks)
    for i in range(P - 1, total - 1):
        idx = vis[i]
        logits, _ = model.forward([seq[j] for j in idx], model.new_cache(len(idx)), positions=idx)
        seq.append(int(logits[-1].argmax()))
    return seq[P:]


class _Session:
    """The native session (`qwen_vk.cpp:497-570`) over oracle caches. Caches 0 and 1 are the two
    windows, 2 the sink buffer; `step(i)` processes position i and returns its logits row."""

    def __init__(self, model, mode: str, shard: int, halo: int, sinks: int, positions: int):
        if mode not in MODES:
            raise ValueError(f"unknown mode {mode!r}")
        self.m, self.mode, self.P = model, mode, positions
        full = mode == "full"
        self.S, self.HALO, self.K = (positions, 0, 0) if full else (shard, halo, sinks)
        if self.S <= 0:
            raise ValueError("shard must be positive")
        if mode in ("shadow", "shadow-batch", "reuse") and (self.HALO > self.S or self.K > self.S):
            raise ValueError("shadow/reuse need halo <= shard and sinks <= shard")
        self.W = min(self.S + self.HALO + self.K, positions)
        self.caches = [model.new_cache(self.W), model.new_cache(self.W), model.new_cache(max(1, min(self.K, self.S)))]
        self.seq: List[int] = []
        self.cur, self.slot, self.slot2 = 0, 0, 0
        self.active = self.sinks_saved = False

    def sinks_of(self, c0: int) -> int:                 # qwen_vk.cpp:279
        return min(self.K, c0 - self.HALO if c0 >= self.HALO else 0)

    def shadowing(self) -> bool:
        return self.mode in ("shadow", "shadow-batch")

    def copy(self, src: int, s0: int, dst: int, d0: int, n: int):   # copy_slots, qwen_vk.cpp:440-453
        a, b = self.caches[src], self.caches[dst]
        for l in range(len(a.keys)):
            b.keys[l][d0:d0 + n] = a.keys[l][s0:s0 + n].clone()
            b.values[l][d0:d0 + n] = a.values[l][s0:s0 + n].clone()

    def run(self, cache: int, i: int, slot: int):
        logits, _ = self.m.forward([self.seq[i]], self.caches[cache], positions=[i], slots=[slot], advance=False)
        return logits[-1]

    def start_shadow(self, nb: int):                    # qwen_vk.cpp:511-515
        ns = self.sinks_of(nb)
        self.copy(2 if self.sinks_saved else self.cur, 0, 1 - self.cur, 0, ns)
        self.slot2, self.active = ns, True

    def step(self, i: int):                             # qwen_vk.cpp:518-565
        S, HALO, K = self.S, self.HALO, self.K
        if i >= self.P:
            raise RuntimeError(f"context full ({self.P} positions)")
        if self.mode != "full" and i > 0 and i % S == 0:
            rebuild = self.mode in ("rebuild", "rebuild-batch")
            if not self.sinks_saved and not rebuild:
                self.copy(self.cur, 0, 2, 0, min(K, S))
                self.sinks_saved = True
            h0, ns = (i - HALO if i >= HALO else 0), self.sinks_of(i)
            if rebuild:                                 # re-run sinks + halo inside the same cache
                self.slot = 0
                for j in list(range(ns)) + list(range(h0, i)):
                    self.run(self.cur, j, self.slot)
                    self.slot += 1
            elif self.shadowing():                      # the shadow window already holds sinks + halo
                if not self.active:
                    self.start_shadow(i)
                self.cur, self.slot, self.active = 1 - self.cur, self.slot2, False
            else:                                       # reuse: sinks + the previous window's halo K/V
                c0p = i - S
                h0p = c0p - HALO if c0p >= HALO else 0
                pre = self.sinks_of(c0p) + (c0p - h0p) if c0p else 0
                self.copy(2, 0, 1 - self.cur, 0, ns)
                self.copy(self.cur, pre + (h0 - c0p), 1 - self.cur, ns, i - h0)
                self.cur, self.slot = 1 - self.cur, ns + (i - h0)
        if self.shadowing() and not self.active and HALO > 0:
            nb = (i // S + 1) * S
            if nb < self.P and i >= nb - HALO:
                self.start_shadow(nb)
        row = self.run(self.cur, i, self.slot)
        self.slot += 1
        if self.active:                                 # the same token in the next shard's window
            self.run(1 - self.cur, i, self.slot2)
            self.slot2 += 1
        return row


@torch.inference_mode()
def session_greedy(model, prompt: Sequence[int], n_new: int, mode: str, shard: int, halo: int, sinks: int,
                   positions: int) -> Tuple[List[int], str]:
    """Greedy tokens of the native session in `mode` (prompt processed position by position, then
    each argmax fed back, `qwen_vk.cpp:567-613`). Returns (tokens, reason): reason "context" when
    the positions run out before n_new tokens."""
    s = _Session(model, mode, shard, halo, sinks, positions)
    s.seq = [int(t) for t in prompt]
    out: List[int] = []
    try:
        row = None
        for i in range(len(s.seq)):
            row = s.step(i)
        while True:
            t = int(row.argmax())
            out.append(t)
            s.seq.append(t)
            if len(out) >= n_new:
                return out, "length"
            row = s.step(len(s.seq) - 1)
    except RuntimeError as exc:
        if not str(exc).startswith("context full"):
            raise
        return out, "context"
