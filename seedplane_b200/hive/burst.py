"""The 16 x 32 independent-request burst over HIVE pull agents, one per GPU (`bench.py --workload burst`).

Every rank (one per GPU) builds the Qwen2-1.5B engine (random-init fp16, seed 0) and runs one
`HiveAgent` (worker id `gpu<rank>`) whose executor generates greedily on that GPU; rank 0 also runs
the loopback `HiveBroker` and drives the burst. Warm-up leases give every worker measured service
times (and capture each GPU's step graph); each timed step then submits the 16 requests as one
`submit_batch`, which splits them by those measurements (identical GPUs: 16 / N each). Requests
partition across GPUs; nothing is exchanged between GPUs.

`value` = generated tokens / the slowest rank's device span (CUDA events around every timed request
on that rank, first start to last end), the max over ranks; `e2e` = the same tokens over rank 0's
wall clock from the first submit to the last result (TCP, JSON and host work included).
"""
from __future__ import annotations

import hashlib
import json
import threading
import time

REQUESTS, NEW_TOKENS, LOW, HIGH = 16, 32, 32, 128
MODEL_ID = "qwen2-1.5b"


def run_burst_bench(args, world, rank, local, ClockSampler, max_over_ranks, barrier, peaks):
    import torch
    import torch.distributed as dist

    from ..config import QWEN2_1_5B
    from ..engine import CudaQwen2
    from ..randinit import burst_prompts, make_weights
    from .agent import GreedyExecutor
    from .pool import HiveAgent, HiveBroker

    cfg = QWEN2_1_5B
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = make_weights(cfg, seed=0, dtype=torch.float16)
    eng = CudaQwen2(cfg, w, device=dev)
    del w
    prompts = burst_prompts(cfg.vocab, REQUESTS, LOW, HIGH, seed=0)

    # device time of this rank's timed requests
    spans = []

    def timer(start: bool):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if start:
            spans.append([ev, None])
        else:
            spans[-1][1] = ev

    base = GreedyExecutor(eng, HIGH + NEW_TOKENS + 1)

    def execute(payload):
        base.timer = timer if payload.get("phase") == "timed" else None
        r = base(payload)
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

    line = None
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

        # warm-up: until every worker has 3 measured leases (and at least args.warmup rounds)
        rounds = 0
        while True:
            futs = broker.submit_batch(payloads("warmup", rounds)[:max(world, 2)], require_profiles=False, **kw)
            for f in futs:
                f.result(timeout=600)
            rounds += 1
            have = [broker.cost_model.estimate(kind="throughput.generate", model=MODEL_ID, worker=f"gpu{r}",
                                               token_budget=NEW_TOKENS) for r in range(world)]
            if rounds >= max(3, args.warmup) and all(h is not None for h in have):
                break
            if rounds > 200:
                raise RuntimeError("warm-up could not measure every worker")
        shas = {}
        assigned = {}
        with ClockSampler(list(range(world))) as clocks:
            t0 = time.perf_counter()
            for step in range(args.steps):
                futs = broker.submit_batch(payloads("timed", step), **kw)
                for f in futs:
                    assigned[f.planned_worker_id] = assigned.get(f.planned_worker_id, 0) + 1
                for f in futs:
                    r = f.result(timeout=600)
                    if shas.setdefault(r["request"], r["token_sha256"]) != r["token_sha256"]:
                        raise RuntimeError(f"request {r['request']}: tokens differ between GPUs / steps")
            wall_s = time.perf_counter() - t0
        broker.close()
        line = {"clocks": clocks.summary(), "wall_s": wall_s, "assigned": assigned,
                "token_sha256": hashlib.sha256(json.dumps([shas[i] for i in sorted(shas)]).encode()).hexdigest()}
    th.join(timeout=600)
    if errors:
        raise errors[0]
    torch.cuda.synchronize(dev)
    span_ms = spans[0][0].elapsed_time(spans[-1][1]) if spans else 0.0
    busy_ms = sum(a.elapsed_time(b) for a, b in spans)
    barrier(world)
    span_max = max_over_ranks(span_ms, world, dev)
    eng.close()
    if rank != 0:
        return None
    tokens = args.steps * REQUESTS * NEW_TOKENS
    prompt_tokens = sum(len(p) for p in prompts)
    return {"metric": "Qwen2-1.5B burst tok/s (16 x 32 requests, HIVE pull agent per GPU)",
            "value": tokens / (span_max / 1000.0), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": span_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{REQUESTS} independent greedy requests x {NEW_TOKENS} new tokens per step, "
                                   f"prompts of uniform-random length in [{LOW}, {HIGH}] (seeded), qwen2-1.5b "
                                   "random-init fp16 weights, one HIVE pull agent per GPU, loopback TCP broker",
                       "parallelism": f"requests partitioned over {world} GPU(s) by measured service time, "
                                      "no collective", "assigned": line["assigned"],
                       "prompt_tokens_per_step": prompt_tokens,
                       "rank0_busy_ms": busy_ms, "l2": "inputs larger than L2: 3.09 GB of weights per step launch"},
            "e2e": {"value": tokens / line["wall_s"], "unit": "tok/s", "h2d_bytes_per_step": prompt_tokens * 4,
                    "d2h_bytes_per_step": REQUESTS * NEW_TOKENS * 4,
                    "note": "rank 0 wall clock: submit_batch to the last result, through the TCP broker"},
            "gpu_launches": args.steps * sum(len(p) + NEW_TOKENS + 1 for p in prompts),
            "clocks": line["clocks"], "token_sha256": line["token_sha256"]}
