#!/usr/bin/env python3
"""Benchmark of the B200 Qwen2 decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|burst]

Workload `decode` (default; the headline configuration): Qwen2-1.5B architecture, random-init
fp16 weights (seed 0, N(0, 0.02), norm gains 1), fp16 KV cache of 4096 slots, a 512-token random
prompt prefilled once, then every step decodes 256 greedy tokens from position 512 (the cache is
rolled back to 512 before each step, so every step does identical work). The metric is decode
tokens per second; with N GPUs every rank runs its own replica (independent requests, no
collective on the data path) and `value` = all ranks' tokens / the slowest rank's time.

The decode line also carries: `e2e` through the drop-in surface (`NativeEngine.generate(ids=...)`
on a checkpoint written to disk: host prompt in, generated tokens out, blocks of device decode);
`burst` (every N: the 16 x 32 HIVE burst on the same engines, tok/s over the wall-clock makespan,
one request per lease, and `burst.batched`: the same burst with each GPU's share decoded as one
batch, runtime request batching);
and at N = 1 `verify` (cfg2: one 16-node tree-verify pass on the Qwen2-0.5B shape), `reference_gpu`
(the reference's own `Qwen2Engine(device='cuda')`, fp16, from `baseline/_ref`, decoding the same
256 tokens after the same prompt on the same GPU) and `cpu_baseline` (the oracle port on the host).

Workload `burst`: the 16 x 32 independent-request burst (prompt lengths uniform in [32, 128]),
requests pulled by one agent per GPU; aggregate tokens / makespan.

`--impl reference` times the reference's CPU algorithm (the oracle port of `Qwen2Engine`) on the
host cores: one greedy token at each of the contexts 512, 576, 640, 704 and 768 per step (the
window the timed decode covers), at the best thread count of a sweep; under torchrun only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import tempfile
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "Qwen2-1.5B decode tok/s"
PROMPT, DECODE, CAPACITY = 512, 256, 4096
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = ",".join(str(g) for g in gpus)
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [s for s in sm if s > 0.5 * (mx or s)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def traffic_per_token():
    """DRAM bytes of one decode step from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "decode_step_qwen2-1.5b_traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_token"])
        except (KeyError, ValueError):
            return None
    return None


# --------------------------------------------------------------------------------------------
def cpu_oracle_sample(cfg, weights, prompt, n_tokens, threads):
    """The oracle port of Qwen2Engine on the host cores: prefill (untimed), then n greedy tokens."""
    from oracle.qwen_oracle import OracleQwen2
    torch.set_num_threads(threads)
    o = OracleQwen2(cfg, weights, kv_fp16=True)
    cache = o.new_cache(len(prompt) + n_tokens + 1)
    logits, cache = o.forward(prompt, cache)
    toks = []
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        toks.append(int(logits[-1].argmax()))
        logits, cache = o.forward([toks[-1]], cache)
    dt = time.perf_counter() - t0
    return n_tokens / dt, toks, dt


def physical_cores():
    try:
        import psutil
        return psutil.cpu_count(logical=False) or os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def thread_counts(n_max: int):
    out, t = [], 1
    while t < n_max:
        out.append(t)
        t *= 2
    return out + [n_max]


def run_reference(args, world, rank):
    if rank != 0:
        return
    from seedplane_b200.config import QWEN2_1_5B
    from seedplane_b200.randinit import make_weights, random_prompt
    from oracle.qwen_oracle import OracleQwen2
    cfg = QWEN2_1_5B
    cores = physical_cores()
    w = make_weights(cfg, seed=0, dtype=torch.float16)
    prompt = random_prompt(cfg.vocab, PROMPT, seed=0)
    torch.set_num_threads(cores)
    o = OracleQwen2(cfg, w, kv_fp16=True)
    del w
    # the cache holds the prompt and 256 more positions (teacher-forced), so a token can be decoded
    # at every context of the timed window; the cost of a decode step depends on its context only
    cache = o.new_cache(CAPACITY)
    o.forward(prompt + random_prompt(cfg.vocab, DECODE, seed=1), cache)
    contexts = [PROMPT + i * DECODE // 4 for i in range(5)]          # 512, 576, 640, 704, 768
    tok = 0

    def step():
        for c in contexts:
            cache.length = c
            o.forward([tok], cache)

    sweep = {}
    for t in thread_counts(cores):
        torch.set_num_threads(t)
        step()                                                       # warm this thread count
        t0 = time.perf_counter()
        step()
        sweep[t] = len(contexts) / (time.perf_counter() - t0)
    best = max(sweep, key=sweep.get)
    torch.set_num_threads(best)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = args.steps * len(contexts) / dt
    model = cpu_model()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "qwen2-1.5b greedy decode at contexts 512..768 after a 512-token prompt "
                                   "(fp16-rounded random-init weights, fp16 K/V), oracle port of Qwen2Engine on the CPU",
                       "tokens_per_step": len(contexts), "contexts": contexts},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": best, "kind": "port",
                             "cpu_model": model, "physical_cores": cores,
                             "thread_sweep_tok_s": {str(k): v for k, v in sweep.items()},
                             "sample": f"one greedy token at each context {contexts} per step (the decode window of "
                                       f"the GPU line), torch {torch.__version__} fp32 on {best} threads (best of "
                                       f"the sweep {sorted(sweep)})"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def write_checkpoint(cfg, weights, directory: Path) -> Path:
    """An HF-named safetensors checkpoint with its config.json (what `NativeEngine` and the
    reference's `Qwen2Engine` load)."""
    from safetensors.torch import save_file
    directory.mkdir(parents=True, exist_ok=True)
    (directory / "config.json").write_text(json.dumps(cfg.to_hf()))
    save_file({k: v.contiguous() for k, v in weights.items()}, str(directory / "model.safetensors"))
    return directory


def native_e2e(ckpt: Path, prompt, want, steps: int, dev):
    """`NativeEngine.generate(ids=prompt)` (the drop-in surface) for DECODE tokens per step: host
    prompt in, the prefill, greedy decode in device blocks, every block's tokens back to the host."""
    from seedplane_b200.native import NativeEngine
    with NativeEngine(ckpt, ctx=CAPACITY, max_new_tokens=DECODE, extra_args=("--device", str(dev))) as ne:
        list(ne.generate(ids=prompt))                                 # warm-up (captures the graphs)
        assert ne.last_tokens == want, "NativeEngine tokens differ from the decode loop"
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(steps):
            list(ne.generate(ids=prompt))
        dt = time.perf_counter() - t0
        assert ne.last_tokens == want
    return steps * DECODE / dt, dt / steps


def reference_gpu(ckpt: Path, prompt, ours, dev):
    """The reference's own PyTorch engine (`seedplane.qwen_engine.Qwen2Engine`, installed unmodified in
    baseline/_ref) on the same GPU, fp16 (its default on CUDA): the prompt, then DECODE greedy tokens
    (contexts 512..767) timed on the wall clock with the device synchronized at both ends."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "seedplane" / "qwen_engine.py").exists():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from seedplane.qwen_engine import Qwen2Engine
    torch.cuda.set_device(dev)
    e = Qwen2Engine(ckpt, device=str(dev))

    def run():
        cache = e.new_cache(CAPACITY)
        logits, cache = e.forward(prompt, cache)
        toks = [int(logits[-1].argmax())]
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(DECODE - 1):
            logits, cache = e.forward([toks[-1]], cache)
            toks.append(int(logits[-1].argmax()))
        torch.cuda.synchronize(dev)
        return toks, time.perf_counter() - t0

    run()
    toks, dt = run()
    match = next((i for i, (a, b) in enumerate(zip(toks, ours)) if a != b), len(toks))
    del e
    torch.cuda.empty_cache()
    return {"value": (DECODE - 1) / dt, "unit": "tok/s", "dtype": "f16 (the reference's CUDA default)",
            "kind": "reference Qwen2Engine(device='cuda') from baseline/_ref, unmodified",
            "sample": f"{DECODE - 1} greedy tokens after the same {PROMPT}-token prompt, one forward per token",
            "tokens_equal_ours_prefix": match}


# --------------------------------------------------------------------------------------------
DECODE_SPECS = {
    # the headline: Qwen2-1.5B fp16, 512-token prompt, 256 greedy tokens per step
    "decode": dict(preset="qwen2-1.5b", fmt="f16", prompt=PROMPT, decode=DECODE, capacity=CAPACITY, metric=METRIC),
    # the int8 target architecture: Qwen2.5-7B shapes, blockwise int8 (32-input blocks, fp16 scales)
    "decode-7b-i8": dict(preset="qwen2.5-7b", fmt="i8", prompt=512, decode=128, capacity=4096,
                         metric="Qwen2.5-7B int8 decode tok/s"),
}


def run_decode(args, world, rank, local):
    """Greedy decode on one GPU per rank (replicas): `value` = decoded tokens of all ranks / the
    slowest rank's device time for the timed steps; each step re-decodes the same tokens after
    the same prompt (the cache length is reset, the prompt's K/V stay)."""
    from seedplane_b200.config import PRESETS
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.randinit import make_int8_blockwise, make_weights, random_prompt
    spec = DECODE_SPECS[args.workload]
    cfg = PRESETS[spec["preset"]]
    PROMPT, DECODE, CAPACITY = spec["prompt"], spec["decode"], spec["capacity"]
    i8 = spec["fmt"] == "i8"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if i8:
        # drawn on the device (a CUDA generator stream): no CPU oracle runs on these weights
        w = make_int8_blockwise(cfg, seed=0, device=str(dev))
        eng = CudaQwen2(cfg, w, device=dev, weight_format="i8")
        del w
        torch.cuda.empty_cache()
    else:
        w = make_weights(cfg, seed=0, dtype=torch.float16)
        eng = CudaQwen2(cfg, w, device=dev)
    prompt = random_prompt(cfg.vocab, PROMPT, seed=0)
    kv = eng.new_kv(CAPACITY)
    _, argmax = eng.forward(kv, prompt, want_logits=False)
    first = int(argmax[-1])
    out = torch.empty(DECODE, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        kv.length = PROMPT
        eng.decode(kv, first, PROMPT, DECODE, out=out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    eng.status()
    tokens_ref = out.cpu().tolist()
    barrier(world)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(list(range(world)) if rank == 0 else [local]) as clocks:
        torch.cuda.synchronize(dev)
        barrier(world)
        t_start.record(stream)
        for _ in range(args.steps):
            step()
        t_end.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
    ms = t_start.elapsed_time(t_end)
    eng.status()
    assert out.cpu().tolist() == tokens_ref, "decode is not deterministic across steps"
    ms_max = max_over_ranks(ms, world, dev)
    total_tokens = args.steps * DECODE * world
    value = total_tokens / (ms_max / 1000.0)
    ms_per_token = ms / (args.steps * DECODE)

    # roofline of the per-token step: one launch of the persistent step kernel per token (the
    # kernel-per-op chain, SEEDPLANE_STEP=chain, launches 5 L + 1 kernels per token instead)
    hbm, peak_kind = peaks()
    avg_ctx = PROMPT + DECODE / 2
    if i8:      # int8 matrices (1 B + a 2-byte scale per 32) and, when tied, the fp16 head
        H, I, V = cfg.hidden, cfg.intermediate, cfg.vocab
        mats = cfg.layers * (cfg.qkv_rows * H + H * H + 3 * I * H) + (0 if cfg.tied_embeddings else V * H)
        w_bytes = cfg.weight_bytes_per_token(0) + mats * (1 + 2 / 32) + (V * H * 2 if cfg.tied_embeddings else 0)
    else:
        w_bytes = cfg.weight_bytes_per_token(2)
    alg_bytes = w_bytes + cfg.kv_bytes_per_position(2) * avg_ctx
    achieved = alg_bytes / (ms_per_token / 1000.0) / 1e9
    traffic = traffic_per_token() if not i8 else None
    step_kernel = os.environ.get("SEEDPLANE_STEP", "step") != "chain"

    # e2e through the drop-in surface: NativeEngine.generate(ids=...) on a checkpoint on disk (fp16
    # path; the int8 line keeps the engine API: NativeEngine loads fp16 bundles)
    want = [first] + tokens_ref[:-1]
    e2e_steps = max(1, min(args.steps, 3))
    # one checkpoint on disk for every rank of the run (rank 0 writes it)
    workdir = Path(tempfile.gettempdir()) / f"seedplane-bench-{os.environ.get('MASTER_PORT', os.getpid())}"
    ckpt = None
    if not i8:
        ckpt = workdir / "ckpt"
        if rank == 0:
            write_checkpoint(cfg, w, ckpt)
        barrier(world)
        e2e_value, e2e_s = native_e2e(ckpt, prompt, want, e2e_steps, dev)
        e2e_h2d, e2e_d2h = PROMPT * 4, DECODE * 4 + 4
        e2e_note = (f"NativeEngine.generate(ids=prompt) per step: host ids in, prefill, {DECODE} greedy tokens "
                    f"(device decode blocks of 32, each block's tokens to the host), wall clock")
    else:
        from seedplane_b200.qwen_engine import KVCache   # noqa: F401
        host_prompt = torch.tensor(prompt, dtype=torch.int32).pin_memory()
        host_out = torch.empty(DECODE, dtype=torch.int32).pin_memory()
        dev_prompt = torch.empty(PROMPT, dtype=torch.int32, device=dev)

        def e2e_step():
            kv.length = 0
            dev_prompt.copy_(host_prompt, non_blocking=True)
            _, am = eng.forward(kv, dev_prompt, want_logits=False)
            first_tok = int(am[-1])
            eng.decode(kv, first_tok, PROMPT, DECODE - 1, out=out[1:])
            out[0] = first_tok
            host_out.copy_(out, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        e2e_step()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        assert host_out.tolist() == want, "public-API tokens differ from the decode loop"
        e2e_value = DECODE / e2e_s
        e2e_h2d, e2e_d2h = PROMPT * 4, DECODE * 4 + 4
        e2e_note = f"engine API per step: pinned prompt H2D, prefill, {DECODE}-token decode, tokens D2H"
    e2e_value = world * DECODE / max_over_ranks(DECODE / e2e_value, world, dev)

    # the 16 x 32 HIVE burst on these engines (every rank; fp16 headline only)
    burst = None
    if not i8 and not args.no_burst:
        from seedplane_b200.hive.burst import burst_on_engine
        burst = burst_on_engine(eng, 2, 3, world, rank, local, ClockSampler, max_over_ranks, barrier)
        # the same burst with runtime request batching: each GPU's share decoded as one batch
        batched = burst_on_engine(eng, 3, 3, world, rank, local, ClockSampler, max_over_ranks, barrier, batched=True)
        if burst is not None:
            # requests whose tokens equal the one-request-per-lease run (a request may part from it at
            # a near-tie of the oracle's logits: the two paths sum in different orders)
            batched["requests_equal_one_per_lease"] = sum(
                x == y for x, y in zip(batched["request_sha256"], burst["request_sha256"]))
            burst["batched"] = batched

    line = None
    if rank == 0:
        L = cfg.layers
        wdesc = "blockwise-int8 (32-input blocks, fp16 scales)" if i8 else "fp16"
        line = {"metric": spec["metric"], "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(3, args.warmup), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "i8xf16" if i8 else "f16", "data": "synthetic",
                "config": {"workload": f"{cfg.name} greedy decode: {DECODE} tokens per step after a {PROMPT}-token "
                                       f"prompt, random-init {wdesc} weights (seed 0), fp16 KV cache",
                           "decode_tokens_per_step": DECODE, "prompt": PROMPT, "kv_capacity": CAPACITY,
                           "weights": wdesc, "accumulate": "fp32", "kv": "fp16",
                           "parallelism": f"replicas x{world} (independent requests, no collective)",
                           "l2": f"inputs larger than L2: {w_bytes / 1e9:.2f} GB of weights streamed per token",
                           "ms_per_token": ms_per_token},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "traffic": traffic,
                             "kernel": ("k_step: persistent per-token decode kernel, one launch per token"
                                        if step_kernel else "one decode step: the GEMV / attention kernel chain"),
                             "algorithmic_bytes_per_launch": alg_bytes, "peak_kind": peak_kind},
                "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": e2e_h2d,
                        "d2h_bytes_per_step": e2e_d2h, "note": e2e_note, "ms_per_step": 1000.0 * e2e_s},
                "gpu_launches": args.steps * (DECODE * (1 if step_kernel else 5 * L + 1) + 1),
                "clocks": clocks.summary(),
                "token_sha256": __import__("hashlib").sha256(json.dumps(tokens_ref).encode()).hexdigest()}
        if i8:
            line["cpu_baseline"] = None
            line["cpu_baseline_note"] = ("not run: the oracle needs the 7B checkpoint dequantized to fp32 (28 GB) "
                                         "in host memory; int8 parity is covered by the tests on smaller shapes")
        if burst is not None:
            line["burst"] = burst
        if world == 1 and not i8 and not args.no_extras:
            line["verify"] = verify_measure(dev, args)
            line["reference_gpu"] = reference_gpu(ckpt, prompt, want, dev)
        if i8:
            pass
        elif world == 1 and not args.no_cpu_baseline:
            threads = physical_cores()
            n = 200    # about 10 s of CPU work on a 16-core host
            val, toks, dt = cpu_oracle_sample(cfg, w, prompt, n, threads)
            line["cpu_baseline"] = {"value": val, "unit": "tok/s", "cores": threads, "kind": "port",
                                    "sample": f"{n} greedy tokens after the same 512-token prompt (prefill "
                                              f"untimed), oracle port fp32 on {threads} threads, {dt:.1f} s",
                                    "tokens_match_gpu": toks == [first] + tokens_ref[:n - 1],
                                    "cpu_model": cpu_model()}
    eng.close()
    barrier(world)
    if rank == 0:
        import shutil
        shutil.rmtree(workdir, ignore_errors=True)
    return line


def verify_measure(dev, args):
    """One batched verify pass of the cfg2 tree (Qwen2-0.5B-shaped fp16 target, a 128-token prompt, 16
    nodes of branching 4, 2, 1, 1 at depth 4): device microseconds per pass (CUDA events over the
    replays of its graph), and the host-side figure with the tree sent and the argmaxes read back."""
    import random
    from seedplane_b200.config import QWEN2_0_5B
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.randinit import make_weights, random_prompt
    cfg = QWEN2_0_5B
    torch.cuda.set_device(dev)
    w = make_weights(cfg, seed=0, dtype=torch.float16)
    eng = CudaQwen2(cfg, w, device=dev)
    del w
    prompt = random_prompt(cfg.vocab, 128, seed=0)
    kv = eng.new_kv(1024)
    eng.forward(kv, prompt, want_logits=False)
    # branching [4, 2, 1, 1] cut to 16 nodes in breadth-first order
    rng = random.Random(0)
    tokens, parents, level = [], [], [-1]
    for width in (4, 2, 1, 1):
        nxt = []
        for par in level:
            for _ in range(width):
                if len(tokens) < 16:
                    tokens.append(rng.randrange(cfg.vocab))
                    parents.append(par)
                    nxt.append(len(tokens) - 1)
        level = nxt
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        am, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
    torch.cuda.synchronize(dev)
    eng.status()
    ref = am.cpu().tolist()
    reps = max(10, args.steps * 20)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler([dev.index]) as clocks:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(reps):
            am, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
        e1.record(stream)
        torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1000.0 / reps
    assert am.cpu().tolist() == ref, "verify is not deterministic"
    t0 = time.perf_counter()
    for _ in range(reps):
        am, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
        host = am.cpu().tolist()
    e2e_us = (time.perf_counter() - t0) * 1e6 / reps
    eng.status()
    eng.close()
    w_bytes = cfg.weight_bytes_per_token(2)
    flops = 2.0 * w_bytes / 2 * len(tokens)
    return {"metric": "tree verify us (16 nodes, Qwen2-0.5B-shaped target)", "value": us, "unit": "us",
            "e2e_us": e2e_us, "nodes": len(tokens), "prompt": len(prompt), "reps": reps,
            "tensor_tflops": flops / (us * 1e-6) / 1e12, "weights_gbs": w_bytes / (us * 1e-6) / 1e9,
            "kernel": "batched pass: k_mcol (tcgen05 multi-column GEMM) + norm / attention kernels, one graph",
            "argmax": host, "clocks": clocks.summary()}


def run_verify(args, world, rank, local):
    """Tree-verify latency (the cfg2 shapes) as the line's own metric: `value` = microseconds per
    verify pass (device, CUDA events on the stream); `e2e` adds the host side: tree arrays to the
    device and the 16 argmaxes back."""
    dev = torch.device("cuda", local)
    v = verify_measure(dev, args)
    if rank != 0:
        return None
    return {"metric": v["metric"], "value": v["value"], "unit": "us",
            "n_gpus": 1, "steps": v["reps"], "warmup": max(3, args.warmup), "ms_per_step": v["value"] / 1000.0,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "one batched verify pass of a 16-node depth-4 draft tree (branching 4,2,1,1 cut "
                                   "to 16) after a 128-token prompt, qwen2-0.5b random-init fp16 target",
                       "nodes": v["nodes"], "prompt": v["prompt"], "tensor_tflops": v["tensor_tflops"],
                       "weights_gbs": v["weights_gbs"], "l2": "inputs larger than L2: 0.99 GB of weights per pass"},
            "e2e": {"value": v["e2e_us"], "unit": "us", "h2d_bytes_per_step": v["nodes"] * 16,
                    "d2h_bytes_per_step": v["nodes"] * 4},
            "clocks": v["clocks"], "argmax": v["argmax"]}


def run_speculative(args, world, rank, local):
    """cfg2: greedy speculative decoding with a Qwen2-0.5B-shaped fp16 target and its first two
    layers as the drafter (+ final norm and LM head), 16-node trees of branching 4, 2, 1, 1, a
    128-token prompt, 64 output tokens. `value` = output tokens per second of the whole loop (wall
    clock, host included); the line also carries the device time per verify pass, the accepted
    draft tokens per round, and whether the tokens equal the target's own greedy decoding."""
    from seedplane_b200.config import QWEN2_0_5B
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.randinit import make_weights, random_prompt, truncate
    from seedplane_b200.speculative import speculative_generate
    from dataclasses import replace
    cfg = QWEN2_0_5B
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = make_weights(cfg, seed=0, dtype=torch.float16)
    target = CudaQwen2(cfg, w, device=dev)
    drafter = CudaQwen2(replace(cfg, layers=2, name="qwen2-0.5b-draft2"), truncate(w, cfg, 2), device=dev)
    del w
    prompt = random_prompt(cfg.vocab, 128, seed=0)
    n_out = 64
    # the target's own greedy tokens (prefill + device decode loop)
    kv = target.new_kv(512)
    _, am = target.forward(kv, prompt, want_logits=False)
    first = int(am[-1])
    rest, _ = target.decode(kv, first, len(prompt), n_out - 1)
    greedy = [first] + rest.tolist()
    kv.close()
    for _ in range(max(1, args.warmup)):
        speculative_generate(target, drafter, prompt, n_out)
    torch.cuda.synchronize(dev)
    times, stats = [], None
    with ClockSampler([local]) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            toks, stats = speculative_generate(target, drafter, prompt, n_out)
            torch.cuda.synchronize(dev)
            times.append(time.perf_counter() - t0)
    target.status()
    drafter.status()
    target.close()
    drafter.close()
    if rank != 0:
        return None
    best = min(times)
    return {"metric": "Qwen2-0.5B speculative greedy tok/s (16-node tree verify, 2-layer drafter)",
            "value": n_out / best, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": max(1, args.warmup), "ms_per_step": 1000 * best, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "cfg2: qwen2-0.5b fp16 target (random-init seed 0), drafter = its first 2 "
                                   "layers, 16-node draft trees (branching 4,2,1,1 kept by cumulative drafter "
                                   "log-probability), 128-token prompt, 64 greedy output tokens",
                       "rounds": stats.rounds, "accepted_per_round": stats.accepted / max(1, stats.rounds),
                       "verify_us_mean": 1000.0 * statistics.mean(stats.verify_ms),
                       "verify_us_median": 1000.0 * statistics.median(stats.verify_ms),
                       "tokens_equal_target_greedy": toks == greedy,
                       "l2": "inputs larger than L2: 0.99 GB of target weights per verify pass"},
            "e2e": {"value": n_out / best, "unit": "tok/s", "h2d_bytes_per_step": 128 * 4,
                    "d2h_bytes_per_step": n_out * 4},
            "clocks": clocks.summary()}


def run_speculative_7b(args, world, rank, local):
    """cfg5: greedy speculative decoding on the Qwen2.5-7B blockwise-int8 target after an 8,192-token
    prompt, with a Qwen2-0.5B-shaped fp16 drafter (its own random init, the target's vocabulary)
    proposing 32-node trees (branching 4, 2, 2, 1, 1, depth 5, kept by cumulative drafter
    log-probability), 128 output tokens. `value` = output tokens per second of the loop (wall clock,
    host included); the line also carries the device time of the 32-node verify passes at this
    context, the accepted draft tokens per round (random weights: ~0, so this measures the loop, not
    a speed-up), whether the tokens equal the target's own greedy decoding, and that decoding's rate
    at the same context."""
    from dataclasses import replace
    from seedplane_b200.config import QWEN2_0_5B, QWEN2_5_7B
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.randinit import make_int8_blockwise, make_weights, random_prompt
    from seedplane_b200.speculative import speculative_generate
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = QWEN2_5_7B
    w = make_int8_blockwise(cfg, seed=0, device=str(dev))
    target = CudaQwen2(cfg, w, device=dev, weight_format="i8")
    del w
    dcfg = replace(QWEN2_0_5B, vocab=cfg.vocab, name="qwen2-0.5b-shaped-drafter")
    dw = make_weights(dcfg, seed=1, dtype=torch.float16)
    drafter = CudaQwen2(dcfg, dw, device=dev)
    del dw
    P, n_out, nodes, branching = 8192, 128, 32, (4, 2, 2, 1, 1)
    prompt = random_prompt(cfg.vocab, P, seed=0)
    cap = P + n_out + 8 * nodes
    # the target's own greedy tokens, and its plain decode rate at this context
    kv = target.new_kv(cap)
    _, am = target.forward(kv, prompt, want_logits=False, last_only=True)
    first = int(am[-1])
    target.decode(kv, first, P, 8)                    # warm the step graph
    kv.length = P
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    rest, _ = target.decode(kv, first, P, n_out - 1)
    e1.record()
    torch.cuda.synchronize(dev)
    decode_ms = e0.elapsed_time(e1) / (n_out - 1)
    greedy = [first] + rest.tolist()
    kv.close()
    speculative_generate(target, drafter, prompt, 8, branching=branching, max_nodes=nodes, capacity=cap)   # warm-up
    torch.cuda.synchronize(dev)
    with ClockSampler([local]) as clocks:
        t0 = time.perf_counter()
        toks, stats = speculative_generate(target, drafter, prompt, n_out, branching=branching, max_nodes=nodes,
                                           capacity=cap)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
    target.status()
    drafter.status()
    target.close()
    drafter.close()
    if rank != 0:
        return None
    return {"metric": "Qwen2.5-7B int8 speculative greedy tok/s (32-node depth-5 tree verify, 0.5B-shaped drafter, "
                      "8,192-token prompt)",
            "value": n_out / wall, "unit": "tok/s", "n_gpus": 1, "steps": 1, "warmup": 1,
            "ms_per_step": 1000 * wall, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 weights, fp32 accumulate", "data": "synthetic",
            "config": {"workload": "cfg5: qwen2.5-7b blockwise-int8 target (random-init seed 0), qwen2-0.5b-shaped "
                                   "fp16 drafter (seed 1, the target's vocabulary), 8,192-token prompt (prefill and "
                                   "the drafter's prefill inside the timed loop), 32-node draft trees, 128 greedy "
                                   "output tokens",
                       "rounds": stats.rounds, "accepted_per_round": stats.accepted / max(1, stats.rounds),
                       "verify_us_mean": 1000.0 * statistics.mean(stats.verify_ms),
                       "verify_us_median": 1000.0 * statistics.median(stats.verify_ms),
                       "tokens_equal_target_greedy": toks == greedy,
                       "target_decode_ms_per_token_at_8k": decode_ms,
                       "l2": "inputs larger than L2: 7.5 GB of int8 weights per decode step"},
            "e2e": {"value": n_out / wall, "unit": "tok/s", "h2d_bytes_per_step": P * 4, "d2h_bytes_per_step": n_out * 4},
            "clocks": clocks.summary()}


def run_burst(args, world, rank, local):
    from seedplane_b200.hive.burst import run_burst_bench
    return run_burst_bench(args, world, rank, local, ClockSampler, max_over_ranks, barrier, peaks)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "decode-7b-i8", "burst", "verify", "speculative",
                                           "speculative-7b-i8"),
                    default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-burst", action="store_true", help="leave the HIVE burst out of the decode line")
    ap.add_argument("--no-extras", action="store_true",
                    help="leave the verify and reference_gpu objects out of the decode line")
    args = ap.parse_args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run = {"burst": run_burst, "verify": run_verify, "speculative": run_speculative,
               "speculative-7b-i8": run_speculative_7b}.get(args.workload, run_decode)
        line = run(args, world, rank, local)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
