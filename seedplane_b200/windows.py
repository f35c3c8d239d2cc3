"""Shard-window attention on the B200 engine: SeedPlane's `ShardPlan` and the native session that
decodes under it.

A long sequence is cut into shards of S tokens. Position i of the shard that starts at c0 attends
to its window only: the first `sinks` tokens of the sequence (fewer when the halo reaches back to
them), the H halo tokens before c0, and its own shard up to itself, all with their original RoPE
positions (`seedplane/engine.py:1-33`).

The engine needs no attention mask for this: a window IS a KV cache of W = S + H + sinks slots
(at most the session's positions), each token written at the next free slot with its original
position, and the step kernel and the batched pass attend to every slot up to their own. The
session moves between windows at shard boundaries the way the reference's native session does
(`native/vulkan_decode/qwen_vk.cpp:497-570`), in one of its modes:

* `full`          -- one window over all positions (ordinary attention).
* `rebuild`       -- at a boundary, the sinks and the halo are re-run one token at a time at the
                     start of the same cache (exact).
* `rebuild-batch` -- the same re-run as one batched pass (exact).
* `shadow`        -- the last H tokens of a shard are also written into a second cache that
                     already holds the next window's sinks; at the boundary the caches swap
                     (exact). The reference runs both windows in one two-column step; here the
                     shadow's copy of a token is written right after the token's own step.
* `shadow-batch`  -- the shadow window's tokens are written in batches (exact; the reference's
                     default).
* `reuse`         -- at a boundary the halo's K/V are copied from the previous window (computed
                     with that window's context: an approximation, fast).

The K/V of the sink tokens are saved from the first window into a small cache of their own at
the first boundary (`qwen_vk.cpp:524`), and copied into each new window with `sp_kv_copy`.

Decoding stays on the device in blocks (`sp_decode`); a block never crosses a boundary or the
start of a shadow window, so the host acts only at those points.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

MODES = ("full", "rebuild", "rebuild-batch", "shadow", "shadow-batch", "reuse")
DEFAULT_MODE = "shadow-batch"            # qwen_vk.cpp:257


@dataclass
class ShardPlan:
    """`seedplane.engine.ShardPlan` (`engine.py:16-33`): S tokens per shard, H halo tokens borrowed
    from the previous shard, `sinks` first tokens visible to every shard (0 = off)."""
    shard: int = 512
    halo: int = 256
    sinks: int = 4

    def __post_init__(self):
        if self.shard <= 0:
            raise ValueError("shard must be greater than zero")
        if self.halo < 0:
            raise ValueError("halo must be non-negative")
        if self.sinks < 0:
            raise ValueError("sinks must be non-negative")

    def windows(self, L):
        """(core_start, core_end, token indices the window reads) for a sequence of L tokens."""
        if L < 0:
            raise ValueError("sequence length must be non-negative")
        c0 = 0
        while c0 < L:
            c1 = min(L, c0 + self.shard)
            h0 = max(0, c0 - self.halo)
            first = list(range(min(self.sinks, h0)))
            yield c0, c1, np.array(first + list(range(h0, c1)), dtype=np.int64)
            c0 += self.shard


class WindowSession:
    """One growing token sequence decoded under a shard plan on one engine (`CudaQwen2`).

    `seq` holds the session's tokens, `done` how many of them have been processed (their K/V are
    in a window). `catch_up()` processes every pending token; `decode_block(n)` runs up to n greedy
    steps on the device from the one pending token and `commit_block(k)` keeps the first k of them
    (the caller cuts at a stop token). A position at or past `positions` raises
    RuntimeError("context full (...)"), like the reference session."""

    def __init__(self, engine, mode: str = "full", plan: Optional[ShardPlan] = None, positions: Optional[int] = None):
        if mode not in MODES:
            raise ValueError(f"unknown attention mode {mode!r} (one of {', '.join(MODES)})")
        cfg = engine.cfg
        P = int(positions if positions is not None else cfg.max_positions)
        if P < 1 or P > cfg.max_positions:
            raise ValueError(f"positions must be in [1, {cfg.max_positions}]")
        plan = plan if plan is not None else ShardPlan()
        self.engine, self.mode, self.P = engine, mode, P
        self.full = mode == "full"
        self.S, self.H, self.K = (P, 0, 0) if self.full else (plan.shard, plan.halo, plan.sinks)
        if not self.full and mode not in ("rebuild", "rebuild-batch") and (self.H > self.S or self.K > self.S):
            raise ValueError("shadow/reuse need halo <= shard and sinks <= shard")     # qwen_vk.cpp:297
        self.W = min(self.S + self.H + self.K, P)
        self.rebuild = mode in ("rebuild", "rebuild-batch")
        self.shadowing = mode in ("shadow", "shadow-batch")
        two = mode in ("shadow", "shadow-batch", "reuse")
        self.caches = [engine.new_kv(self.W)] + ([engine.new_kv(self.W)] if two else [])
        n_sink = min(self.K, self.S)
        self.sink_kv = engine.new_kv(n_sink) if (two and n_sink > 0) else None
        self.reset()

    # ---- state ---------------------------------------------------------------------------------
    def reset(self):
        self.seq: List[int] = []
        self.done = 0
        self.cur = 0
        self.slot = self.slot2 = 0
        self.active = self.sinks_saved = False
        self._block = None

    @property
    def plan(self) -> dict:
        return {"shard": self.S, "halo": self.H, "sinks": self.K}

    def sinks_of(self, c0: int) -> int:
        """Sink tokens of the window whose shard starts at c0 (`qwen_vk.cpp:279`)."""
        return min(self.K, c0 - self.H if c0 >= self.H else 0)

    def close(self):
        for kv in self.caches + ([self.sink_kv] if self.sink_kv is not None else []):
            kv.close()
        self.caches, self.sink_kv = [], None

    # ---- engine calls ----------------------------------------------------------------------------
    def _forward(self, kv, ids: Sequence[int], positions: Sequence[int], slot: int, want_logits=False):
        kv.length = slot
        logits, am = self.engine.forward(kv, torch.tensor(list(ids), dtype=torch.int32),
                                         positions=list(positions), want_logits=want_logits, last_only=True)
        return logits, am

    def _copy(self, src, s0: int, dst, d0: int, n: int):
        if n > 0:
            self.engine.kv_copy(src, s0, dst, d0, n)

    # ---- window moves (qwen_vk.cpp:511-548), run before position i is processed -----------------
    def _start_shadow(self, nb: int):
        ns = self.sinks_of(nb)
        self._copy(self.sink_kv if self.sinks_saved else self.caches[self.cur], 0, self.caches[1 - self.cur], 0, ns)
        self.slot2, self.active = ns, True

    def _transition(self, i: int):
        if i >= self.P:
            raise RuntimeError(f"context full ({self.P} positions)")
        S, H = self.S, self.H
        if not self.full and i > 0 and i % S == 0:
            if not self.sinks_saved and not self.rebuild:
                self._copy(self.caches[self.cur], 0, self.sink_kv, 0, min(self.K, S))
                self.sinks_saved = True
            h0, ns = (i - H if i >= H else 0), self.sinks_of(i)
            if self.rebuild:                     # re-run the sinks and the halo inside the new window
                items = list(range(ns)) + list(range(h0, i))
                kv = self.caches[self.cur]
                if self.mode == "rebuild-batch":
                    if items:
                        self._forward(kv, [self.seq[j] for j in items], items, 0)
                else:
                    for s, j in enumerate(items):
                        self._forward(kv, [self.seq[j]], [j], s)
                self.slot = len(items)
            elif self.shadowing:                 # the shadow window already holds sinks + halo
                if not self.active:
                    self._start_shadow(i)
                self.cur, self.slot, self.active = 1 - self.cur, self.slot2, False
            else:                                # reuse: sinks, then the previous window's halo K/V
                c0p = i - S
                h0p = c0p - H if c0p >= H else 0
                pre = self.sinks_of(c0p) + (c0p - h0p) if c0p else 0
                other = self.caches[1 - self.cur]
                self._copy(self.sink_kv, 0, other, 0, ns)
                self._copy(self.caches[self.cur], pre + (h0 - c0p), other, ns, i - h0)
                self.cur, self.slot = 1 - self.cur, ns + (i - h0)
        if self.shadowing and not self.active and H > 0:
            nb = (i // S + 1) * S
            if nb < self.P and i >= nb - H:
                self._start_shadow(nb)

    def _next_transition(self, i: int) -> int:
        """The first position after i at which the session acts before processing it."""
        if self.full:
            return self.P
        nb = (i // self.S + 1) * self.S
        nxt = nb
        if self.shadowing and not self.active and self.H > 0 and nb < self.P and nb - self.H > i:
            nxt = nb - self.H
        return min(nxt, self.P)

    # ---- processing ----------------------------------------------------------------------------------
    def _shadow_append(self, i0: int, n: int):
        if self.active and n > 0:
            self._forward(self.caches[1 - self.cur], self.seq[i0:i0 + n], range(i0, i0 + n), self.slot2)
            self.slot2 += n

    def catch_up(self, want_logits: bool = False):
        """Process every pending token; returns (logits [1, V] of the last one or None, its argmax)."""
        if self._block is not None:
            raise RuntimeError("a decode block is not committed")
        if self.done >= len(self.seq):
            raise RuntimeError("no pending token")
        logits, last = None, None
        while self.done < len(self.seq):
            i = self.done
            self._transition(i)
            n = min(len(self.seq) - i, self._next_transition(i) - i)
            end = i + n == len(self.seq)
            logits, am = self._forward(self.caches[self.cur], self.seq[i:i + n], range(i, i + n), self.slot,
                                       want_logits=want_logits and end)
            self.slot += n
            self._shadow_append(i, n)
            self.done = i + n
            if end:
                last = int(am[-1])
        return logits, last

    def decode_block(self, n_max: int, want_logits: bool = False):
        """Up to n_max greedy steps on the device from the pending token seq[done] (the block stops
        before the next window move). Returns (argmax of every step int32 [n], logits of the last
        step or None); `commit_block` must follow."""
        if self._block is not None:
            raise RuntimeError("a decode block is not committed")
        if self.done != len(self.seq) - 1:
            raise RuntimeError("decode_block needs exactly one pending token")
        i = self.done
        self._transition(i)
        n = max(1, min(int(n_max), self._next_transition(i) - i))
        kv = self.caches[self.cur]
        kv.length = self.slot
        out, logits = self.engine.decode(kv, self.seq[i], i, n, want_logits=want_logits)
        self._block = (i, self.slot, n)
        return out, logits

    def commit_block(self, k: int):
        """Keep the first k steps of the last block: positions done .. done + k - 1 stay processed
        (the fed token and the first k - 1 argmaxes, which the caller has appended to `seq`)."""
        if self._block is None:
            raise RuntimeError("no decode block to commit")
        i, slot, n = self._block
        if not 1 <= k <= n or len(self.seq) < i + k:
            raise ValueError("commit outside the block")
        self._block = None
        self.slot = slot + k
        self.caches[self.cur].length = self.slot
        self._shadow_append(i, k)
        self.done = i + k
