"""Measured service-cost model of HIVE work (`seedplane/hive/cost.py:1-99` of the reference).

Per (kind, model, worker, size bucket, batch bucket, load bucket) it keeps the last `history`
durations; an estimate needs `min_samples` of them and reports the median and the nearest-rank
95th percentile. Size and batch buckets are ceil(log2(value)) (0 for values <= 1); the load
bucket is int(10 * load) clamped to 0..9.
"""
from __future__ import annotations

import math
import statistics
import threading
from collections import defaultdict, deque
from dataclasses import dataclass
from typing import Optional


def log2_bucket(value) -> int:
    return 0 if value <= 1 else int(math.ceil(math.log2(value)))


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


class MeasuredCostModel:
    def __init__(self, *, history: int = 128, min_samples: int = 3):
        if history < 1 or min_samples < 1:
            raise ValueError("history and min_samples must be positive")
        self.history = int(history)
        self.min_samples = int(min_samples)
        self._samples = defaultdict(lambda: deque(maxlen=self.history))
        self._lock = threading.Lock()

    @staticmethod
    def key(kind, model, worker, token_budget, batch_size=1, load=0.0) -> CostKey:
        return CostKey(str(kind), str(model), str(worker), log2_bucket(token_budget), log2_bucket(batch_size),
                       min(9, max(0, int(load * 10))))

    def observe(self, *, kind, model, worker, token_budget, duration_ms, batch_size=1, load=0.0) -> CostKey:
        d = float(duration_ms)
        if not (math.isfinite(d) and d > 0):
            raise ValueError("duration_ms must be finite and positive")
        k = self.key(kind, model, worker, token_budget, batch_size, load)
        with self._lock:
            self._samples[k].append(d)
        return k

    def estimate(self, *, kind, model, worker, token_budget, batch_size=1, load=0.0) -> Optional[CostEstimate]:
        k = self.key(kind, model, worker, token_budget, batch_size, load)
        with self._lock:
            values = sorted(self._samples.get(k, ()))
        if len(values) < self.min_samples:
            return None
        rank95 = max(1, math.ceil(0.95 * len(values)))
        return CostEstimate(statistics.median(values), values[rank95 - 1], len(values))

    @staticmethod
    def choose_lease_tokens(*, throughput_tokens_s, fixed_overhead_ms, max_fixed_fraction=0.2, min_tokens=1,
                            max_tokens=4096):
        """Smallest lease (tokens) whose fixed overhead is at most `max_fixed_fraction` of its time."""
        rate, fixed, frac = float(throughput_tokens_s), float(fixed_overhead_ms), float(max_fixed_fraction)
        if rate <= 0 or fixed < 0 or not 0 < frac < 1:
            raise ValueError("invalid throughput, overhead, or fixed-cost fraction")
        if fixed == 0:
            return int(min_tokens)
        tokens = math.ceil(rate * (fixed * (1.0 - frac) / frac) / 1000.0)
        return int(min(max_tokens, max(min_tokens, tokens)))

    def snapshot(self):
        with self._lock:
            return {k: tuple(v) for k, v in self._samples.items()}
