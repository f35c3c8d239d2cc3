"""Makespan-optimal split of identical independent requests (`seedplane/hive/scheduler.py:12-59`).

With per-request service times s_w, the smallest batch deadline D is the least value of the form
k * s_w at which the workers can finish N requests: sum_w floor(D / s_w) >= N. The workers are
then filled fastest first (ties by name) with min(remaining, floor(D / s_w)) requests, so a slow
worker may get none and adding a worker never worsens the predicted makespan.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict

_EPS = 1e-9


@dataclass(frozen=True)
class BatchPlan:
    assignments: Dict[str, int]
    predicted_makespan_ms: float


def plan_homogeneous_batch(task_count, worker_service_ms) -> BatchPlan:
    n = int(task_count)
    service = {str(w): float(ms) for w, ms in worker_service_ms.items()}
    if n < 0 or not service:
        raise ValueError("task_count must be non-negative and worker profiles non-empty")
    if any(not math.isfinite(ms) or ms <= 0 for ms in service.values()):
        raise ValueError("worker service estimates must be finite and positive")
    if n == 0:
        return BatchPlan({w: 0 for w in service}, 0.0)

    def capacity(deadline):
        return sum(int((deadline + _EPS * deadline) // s) for s in service.values())

    candidates = sorted({k * s for s in service.values() for k in range(1, n + 1)})
    lo, hi = 0, len(candidates) - 1          # the fastest worker alone meets candidates[...n * s_min]
    while lo < hi:
        mid = (lo + hi) // 2
        if capacity(candidates[mid]) >= n:
            hi = mid
        else:
            lo = mid + 1
    deadline = candidates[lo]
    plan = {w: 0 for w in service}
    left = n
    for w, s in sorted(service.items(), key=lambda kv: (kv[1], kv[0])):
        take = min(left, int((deadline + _EPS * deadline) // s))
        plan[w] = take
        left -= take
        if left == 0:
            break
    if left:
        raise RuntimeError("internal error: the batch deadline is infeasible")
    return BatchPlan(plan, max(plan[w] * s for w, s in service.items()))
