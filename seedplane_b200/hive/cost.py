"""Measured service-time model of HIVE work: the interface of the reference's
`seedplane/hive/cost.py` (`CostKey`, `CostEstimate`, `MeasuredCostModel`), a window design of its own.

Each key keeps a sliding window of its most recent durations twice: in arrival order (to know which
sample leaves the window next) and sorted (so a quantile is an index, not a sort). `estimate` then
reads the median and the nearest-rank 95th percentile straight from the sorted copy. Keys bucket
the request size and batch size on a log2 scale (so nearby sizes share history) and the load in
tenths.
"""
from __future__ import annotations

import bisect
import math
import threading
from collections import deque
from dataclasses import dataclass
from typing import Dict, Optional, Tuple


def log2_bucket(value) -> int:
    """0 for sizes up to 1, else the exponent of the next power of two (3 -> 2, 4 -> 2, 5 -> 3)."""
    v = float(value)
    if v <= 1.0:
        return 0
    m, e = math.frexp(v)              # v = m * 2^e, 0.5 <= m < 1
    return e - 1 if m == 0.5 else e


def load_bucket(load) -> int:
    """Load in tenths, clamped to 0 .. 9."""
    return min(9, max(0, int(float(load) * 10)))


@dataclass(frozen=True)
class CostKey:
    kind: str
    model: str
    worker: str
    size_bucket: int
    batch_bucket: int = 0
    load_bucket: int = 0


@dataclass(frozen=True)
class CostEstimate:
    p50_ms: float
    p95_ms: float
    samples: int


class _Window:
    """The last `cap` durations of one key, in arrival order and sorted."""

    __slots__ = ("arrivals", "ordered", "cap")

    def __init__(self, cap: int):
        self.cap = cap
        self.arrivals: deque = deque()
        self.ordered: list = []

    def push(self, d: float) -> None:
        if len(self.arrivals) == self.cap:
            old = self.arrivals.popleft()
            del self.ordered[bisect.bisect_left(self.ordered, old)]
        self.arrivals.append(d)
        bisect.insort(self.ordered, d)

    def median(self) -> float:
        n = len(self.ordered)
        mid = n // 2
        return self.ordered[mid] if n % 2 else 0.5 * (self.ordered[mid - 1] + self.ordered[mid])

    def nearest_rank(self, q: float) -> float:
        """The smallest sample with at least a fraction q of the window at or below it."""
        rank = max(1, math.ceil(q * len(self.ordered)))
        return self.ordered[rank - 1]


class MeasuredCostModel:
    """Per-key windows of measured durations (ms). An estimate needs `min_samples` of them."""

    def __init__(self, *, history: int = 128, min_samples: int = 3):
        if history < 1 or min_samples < 1:
            raise ValueError("history and min_samples must be positive")
        self.history = int(history)
        self.min_samples = int(min_samples)
        self._windows: Dict[CostKey, _Window] = {}
        self._mutex = threading.Lock()

    @staticmethod
    def key(kind, model, worker, token_budget, batch_size=1, load=0.0) -> CostKey:
        return CostKey(kind=str(kind), model=str(model), worker=str(worker), size_bucket=log2_bucket(token_budget),
                       batch_bucket=log2_bucket(batch_size), load_bucket=load_bucket(load))

    def observe(self, *, kind, model, worker, token_budget, duration_ms, batch_size=1, load=0.0) -> CostKey:
        d = float(duration_ms)
        if math.isnan(d) or math.isinf(d) or d <= 0.0:
            raise ValueError(f"a measured duration must be a positive finite number of ms, got {duration_ms!r}")
        k = self.key(kind, model, worker, token_budget, batch_size, load)
        with self._mutex:
            w = self._windows.get(k)
            if w is None:
                w = self._windows[k] = _Window(self.history)
            w.push(d)
        return k

    def estimate(self, *, kind, model, worker, token_budget, batch_size=1, load=0.0) -> Optional[CostEstimate]:
        k = self.key(kind, model, worker, token_budget, batch_size, load)
        with self._mutex:
            w = self._windows.get(k)
            if w is None or len(w.ordered) < self.min_samples:
                return None
            return CostEstimate(p50_ms=w.median(), p95_ms=w.nearest_rank(0.95), samples=len(w.ordered))

    @staticmethod
    def choose_lease_tokens(*, throughput_tokens_s, fixed_overhead_ms, max_fixed_fraction=0.2, min_tokens=1,
                            max_tokens=4096) -> int:
        """The smallest lease, in tokens, whose fixed overhead is at most `max_fixed_fraction` of the
        lease's total time. A lease of n tokens at r tokens/s spends 1000 n / r ms on work; the
        overhead share f0 / (f0 + 1000 n / r) <= f holds from n = r f0 (1 / f - 1) / 1000 on. The
        answer is clamped to [min_tokens, max_tokens]."""
        rate, f0, share = float(throughput_tokens_s), float(fixed_overhead_ms), float(max_fixed_fraction)
        if not (rate > 0.0 and f0 >= 0.0 and 0.0 < share < 1.0):
            raise ValueError("throughput must be positive, overhead non-negative and the share in (0, 1)")
        if f0 == 0.0:
            return int(min_tokens)
        work_ms = f0 * (1.0 / share - 1.0)
        n = math.ceil(work_ms * rate / 1000.0)
        return int(max(min_tokens, min(max_tokens, n)))

    def snapshot(self) -> Dict[CostKey, Tuple[float, ...]]:
        """Every key's window in arrival order."""
        with self._mutex:
            return {k: tuple(w.arrivals) for k, w in self._windows.items()}
