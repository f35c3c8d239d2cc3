"""The 16 x 32 independent-request burst over HIVE pull agents, one per GPU (`bench.py --workload burst`).

Every rank (one per GPU) builds the Qwen2-1.5B engine (random-init fp16, seed 0) and runs one
`HiveAgent` (worker id `gpu<rank>`) whose executor generates greedily on that GPU; rank 0 also runs
the loopback `HiveBroker` and drives the burst. Warm-up leases give every worker measured service
times (and capture each GPU's step graph); each timed step then submits the 16 requests as one
`submit_batch`, which splits them by those measurements (identical GPUs: 16 / N each). Requests
partition across GPUs; nothing is exchanged between GPUs.

`value` = generated tokens / the makespan on rank 0's wall clock, from the first submit to the last
result (TCP, JSON and host work included: the reference's own burst measure,
`experiments/hive_scaling/benchmark_hive_fleet.py:112`); `device_tok_s` = the same tokens over the
slowest rank's device span (CUDA events around every timed request on that rank, first start to
last end, the max over ranks).

`burst_on_engine` runs the same burst on an engine the caller already built (the decode bench's
replica on every rank) and returns the summary object the bench line carries.
"""
from __future__ import annotations

import hashlib
import json
import threading
import time

REQUESTS, NEW_TOKENS, LOW, HIGH = 16, 32, 32, 128
MODEL_ID = "qwen2-1.5b"


def burst_on_engine(eng, steps, warmup, world, rank, local, ClockSampler, max_over_ranks, barrier, batched=False):
    """The 16 x 32 burst through HIVE on `eng` (this rank's engine); every rank calls it. Returns the
    summary on rank 0 (None elsewhere). `batched`: each GPU's share of a timed step goes out as one
    grouped lease that its agent decodes as one batch (runtime request batching); warm-up leases
    stay single requests, which is what the planner measures."""
    import torch
    import torch.distributed as dist

    from ..randinit import burst_prompts
    from .agent import GreedyExecutor
    from .pool import HiveAgent, HiveBroker

    dev = eng.device
    torch.cuda.set_device(dev)
    prompts = burst_prompts(eng.cfg.vocab, REQUESTS, LOW, HIGH, seed=0)
    spans = []                                  # device time of this rank's timed requests

    def timer(start: bool):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if start:
            spans.append([ev, None])
        else:
            spans[-1][1] = ev

    base = GreedyExecutor(eng, HIGH + NEW_TOKENS + 1)

    def execute(payload):
        items = payload.get("batch")
        phase = (items[0] if items else payload).get("phase")
        base.timer = timer if phase == "timed" else None
        r = base(payload)
        if items is not None:
            for it, res in zip(items, r["batch"]):
                res["request"] = it.get("request")
        else:
            r["request"] = payload.get("request")
        return r

    broker = None
    port = torch.zeros(1, dtype=torch.int64, device=dev)
    if rank == 0:
        broker = HiveBroker(pull_poll_s=0.02).start()
        port[0] = broker.address[1]
    if world > 1:
        dist.broadcast(port, 0)
    agent = HiveAgent("127.0.0.1", int(port.item()), f"gpu{rank}", caps=("generate", "throughput.generate"),
                      models=(MODEL_ID,), execute=execute)
    errors = []

    def run_agent():
        try:
            torch.cuda.set_device(dev)
            agent.run()
        except Exception as exc:              # reported by the rank after the burst
            errors.append(exc)

    th = threading.Thread(target=run_agent, name=f"hive-agent-gpu{rank}", daemon=True)
    th.start()
    info = None
    if rank == 0:
        t_end = time.monotonic() + 300
        while len(broker.workers()) < world and time.monotonic() < t_end:
            time.sleep(0.01)
        if len(broker.workers()) < world:
            raise RuntimeError(f"only {len(broker.workers())} of {world} agents connected")
        kw = dict(model=MODEL_ID, required_caps=("generate",), token_budget=NEW_TOKENS, timeout=600)

        def payloads(phase, step):
            return [{"ids": p, "max_new_tokens": NEW_TOKENS, "request": i, "phase": phase, "step": step}
                    for i, p in enumerate(prompts)]

        # warm-up: until every worker has 3 measured leases (and at least `warmup` rounds)
        rounds = 0
        while True:
            for f in broker.submit_batch(payloads("warmup", rounds)[:max(world, 2)], require_profiles=False, **kw):
                f.result(timeout=600)
            rounds += 1
            have = [broker.cost_model.estimate(kind="throughput.generate", model=MODEL_ID, worker=f"gpu{r}",
                                               token_budget=NEW_TOKENS) for r in range(world)]
            if rounds >= max(3, warmup) and all(h is not None for h in have):
                break
            if rounds > 200:
                raise RuntimeError("warm-up could not measure every worker")
        if batched:                             # the grouped path once (captures each GPU's batch graph)
            for f in broker.submit_batch(payloads("warmup", rounds), group_per_worker=True, **kw):
                f.result(timeout=600)
        shas, assigned, makespans = {}, {}, []
        with ClockSampler(list(range(world))) as clocks:
            for step in range(steps):
                t0 = time.perf_counter()
                futs = broker.submit_batch(payloads("timed", step), group_per_worker=batched, **kw)
                for f in futs:
                    assigned[f.planned_worker_id] = assigned.get(f.planned_worker_id, 0) + 1
                for f in futs:
                    r = f.result(timeout=600)
                    if shas.setdefault(r["request"], r["token_sha256"]) != r["token_sha256"]:
                        raise RuntimeError(f"request {r['request']}: tokens differ between GPUs / steps")
                makespans.append(time.perf_counter() - t0)
        broker.close()
        info = {"clocks": clocks.summary(), "makespans": makespans, "assigned": assigned,
                "token_sha256": hashlib.sha256(json.dumps([shas[i] for i in sorted(shas)]).encode()).hexdigest(),
                "request_sha256": [shas[i] for i in sorted(shas)]}
    th.join(timeout=600)
    if errors:
        raise errors[0]
    torch.cuda.synchronize(dev)
    span_ms = spans[0][0].elapsed_time(spans[-1][1]) if spans else 0.0
    barrier(world)
    span_max = max_over_ranks(span_ms, world, dev)
    if rank != 0:
        return None
    tokens = steps * REQUESTS * NEW_TOKENS
    wall = sum(info["makespans"])
    return {"metric": "burst tok/s (16 x 32 requests, HIVE pull agent per GPU, wall-clock makespan)",
            "batched": bool(batched),
            "value": tokens / wall, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "makespan_ms": [1000.0 * m for m in info["makespans"]],
            "device_tok_s": tokens / (span_max / 1000.0) if span_max > 0 else None,
            "assigned": info["assigned"], "prompt_tokens_per_step": sum(len(p) for p in prompts),
            "token_sha256": info["token_sha256"], "request_sha256": info["request_sha256"], "clocks": info["clocks"],
            "note": "makespan = submit_batch to the last result on rank 0 (loopback TCP broker, JSON, host work "
                    "included); device_tok_s = the same tokens over the slowest rank's device span"}


def run_burst_bench(args, world, rank, local, ClockSampler, max_over_ranks, barrier, peaks):
    """`bench.py --workload burst`: the burst as the line's own metric."""
    import torch
    from ..config import QWEN2_1_5B
    from ..engine import CudaQwen2
    from ..randinit import make_weights
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = make_weights(QWEN2_1_5B, seed=0, dtype=torch.float16)
    eng = CudaQwen2(QWEN2_1_5B, w, device=dev)
    del w
    single = burst_on_engine(eng, args.steps, args.warmup, world, rank, local, ClockSampler, max_over_ranks, barrier)
    b = burst_on_engine(eng, args.steps, args.warmup, world, rank, local, ClockSampler, max_over_ranks, barrier,
                        batched=True)
    eng.close()
    if rank != 0:
        return None
    tokens = args.steps * REQUESTS * NEW_TOKENS
    wall_ms = sum(b["makespan_ms"])
    return {"metric": "Qwen2-1.5B burst tok/s (16 x 32 requests, HIVE pull agent per GPU)",
            "value": b["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": wall_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{REQUESTS} independent greedy requests x {NEW_TOKENS} new tokens per step, "
                                   f"prompts of uniform-random length in [{LOW}, {HIGH}] (seeded), qwen2-1.5b "
                                   "random-init fp16 weights, one HIVE pull agent per GPU, loopback TCP broker; "
                                   "each GPU's share as one grouped lease decoded as a batch",
                       "one_request_per_lease": {"value": single["value"], "makespan_ms": single["makespan_ms"],
                                                 "token_sha256": single["token_sha256"],
                                                 "requests_with_equal_tokens": sum(
                                                     x == y for x, y in zip(single["request_sha256"],
                                                                            b["request_sha256"]))},
                       "parallelism": f"requests partitioned over {world} GPU(s) by measured service time, "
                                      "no collective", "assigned": b["assigned"],
                       "device_tok_s": b["device_tok_s"],
                       "l2": "inputs larger than L2: 3.09 GB of weights per step launch"},
            "e2e": {"value": b["value"], "unit": "tok/s", "h2d_bytes_per_step": b["prompt_tokens_per_step"] * 4,
                    "d2h_bytes_per_step": REQUESTS * NEW_TOKENS * 4, "note": b["note"]},
            "gpu_launches": None, "clocks": b["clocks"], "token_sha256": b["token_sha256"]}
