"""Short decode runs for profiling and launch-mode comparisons.

    python -m seedplane_b200.profile_decode --model qwen2-1.5b --prompt 16 --tokens 8 [--modes graph+pdl,graph,eager+pdl]

Prints, per launch mode, the device time per decoded token (CUDA events) and the host time spent
enqueueing the step launches. With `--modes graph+pdl --repeat 0` it is also the small, bounded
command used under `ncu` (a prefill of `--prompt` tokens and `--tokens` decode steps).
"""
from __future__ import annotations

import argparse
import json
from dataclasses import replace
import os
import time

import torch

from .config import PRESETS
from .randinit import make_int8_blockwise, make_weights, random_prompt

MODES = {"graph+pdl": ("1", "1"), "graph": ("1", "0"), "eager+pdl": ("0", "1"), "eager": ("0", "0")}
# --step chain|step: the kernel-per-op chain or the persistent step kernel


KERNELS = ("qkv", "o", "gate_up", "down")


STEP_OPS = ("qkv", "attn", "o", "gate_up", "down")


def step_trace_summary(t, layers, layers_shown=(0, 1, 13)):
    """Timeline of the persistent step kernel from its per-op, per-CTA stamps (microseconds):
    [0] the CTA reached the op, [1] its dependency was met, [2] input vector ready, [3] op done,
    [4] first weight unit available, [5] all rows finished."""
    import numpy as np
    t0 = t[t > 0].min()
    t = np.where(t > 0, (t - t0) / 1000.0, np.nan)
    rows, prev_done = [], 0.0
    gemv = lambda x: x if True else None
    for k in range(t.shape[0]):
        layer, kind = (k // 5, STEP_OPS[k % 5]) if k < 5 * layers else (-1, "lm_head")
        done = float(np.nanmax(t[k, :, 3]))
        g = kind != "attn"
        med = lambda j: float(np.nanmedian(t[k, :, j])) if g else None
        mx = lambda j: float(np.nanmax(t[k, :, j])) if g else None
        if kind == "attn":       # item CTAs only: [1] QKV ready, [2] staged, [4] computed, [6]/[7] merge
            a = lambda j, f: float(f(t[k, :, j])) if not np.isnan(t[k, :, j]).all() else None
            row = {"k": k, "layer": layer, "kind": kind, "qkv_seen_max": a(1, np.nanmax), "staged_max": a(2, np.nanmax),
                   "scores_max": a(5, np.nanmax), "computed_med": a(4, np.nanmedian), "computed_max": a(4, np.nanmax),
                   "merge_start_max": a(6, np.nanmax), "merge_end_max": a(7, np.nanmax),
                   "done_max": float(np.nanmax(t[k, :, 3])), "since_prev_done": float(np.nanmax(t[k, :, 3])) - prev_done}
            prev_done = row["done_max"]
            if layer in layers_shown:
                rows.append({key: (round(v, 2) if isinstance(v, float) else v) for key, v in row.items()})
            continue
        row = {"k": k, "layer": layer, "kind": kind, "dep_met_max": mx(1), "input_med": med(2),
               "unit0_med": med(4), "rows_med": med(5), "rows_max": mx(5),
               "done_med": float(np.nanmedian(t[k, :, 3])), "done_max": done, "since_prev_done": done - prev_done}
        prev_done = done
        if layer in layers_shown or layer == -1:
            rows.append({key: (round(v, 2) if isinstance(v, float) else v) for key, v in row.items()})
    span = float(np.nanmax(t[:, :, 3]))
    per_layer = [float(np.nanmax(t[5 * l + 4, :, 3]) - (np.nanmax(t[5 * l - 1, :, 3]) if l else 0.0))
                 for l in range(layers)]
    return {"step_span_us": round(span, 1), "layer_us_median": round(float(np.median(per_layer)), 2), "ops": rows}


GEMV_PHASES = ("prologue", "unit_wait", "mma", "epilogue", "signal")
ATTN_PHASES = ("poll_qkv", "stage", "scores", "softmax", "values", "publish_to_merge", "merge")


def step_phase_summary(clk, gt, layers):
    """Median per-CTA phase durations (microseconds, from clock64 at the SM clock) per op kind over
    layers 1 .. L-1: GEMV [0] start [1] input ready [2] first unit [3] MMA done [4] epilogue done
    [5] signalled; attention [0] poll start [1] q/kv seen [2] staged [3] scores [4] softmax
    [5] values done [6] merge start [7] merge end."""
    import numpy as np
    c = clk.astype(np.float64)
    g = gt.astype(np.float64)
    # SM clock from the first and the last layer's QKV op: clock64 cycles per %globaltimer ns
    k1 = 5 * (layers - 1)
    dc, dt = c[k1, :, 0] - c[0, :, 0], g[k1, :, 0] - g[0, :, 0]
    ok = (c[k1, :, 0] > 0) & (c[0, :, 0] > 0) & (dt > 0)
    mhz = float(np.median(dc[ok] / dt[ok])) * 1000.0 if ok.any() else 1965.0
    out = {}
    for j, kind in enumerate(STEP_OPS):
        ks = [5 * l + j for l in range(1, layers)]
        x = c[ks]                                            # [layers - 1, sms, 8]
        names = ATTN_PHASES if kind == "attn" else GEMV_PHASES
        d = {}
        for i, name in enumerate(names):
            a, b = x[:, :, i], x[:, :, i + 1]
            ok = (a > 0) & (b > 0) & (b >= a)
            if ok.any():
                d[name] = round(float(np.median((b - a)[ok])) / mhz, 3)
        out[kind] = d
    out["sm_mhz"] = round(mhz, 1)
    return out


def trace_summary(eng, layers_shown=(0, 1, 13)):
    """Per-GEMV timeline of the last step from the %globaltimer stamps (microseconds)."""
    import ctypes as C
    import numpy as np
    from . import _native as N
    lib = N.load()
    n = lib.sp_trace_read(eng.handle, None, 0)
    if n <= 0:
        return {}
    buf = (C.c_uint64 * n)()
    N.check(0 if lib.sp_trace_read(eng.handle, buf, n) == n else -2)
    sms = torch.cuda.get_device_properties(eng.device).multi_processor_count
    if n == (5 * eng.cfg.layers + 1) * sms * 16:       # persistent step kernel
        raw = np.frombuffer(buf, dtype=np.uint64).reshape(-1, sms, 16)
        out = step_trace_summary(raw[:, :, :8].astype(np.float64), eng.cfg.layers, layers_shown)
        out["phases_us"] = step_phase_summary(raw[:, :, 8:], raw[:, :, :8], eng.cfg.layers)
        return out
    words = 8 + 2 * 24
    t = np.frombuffer(buf, dtype=np.uint64).astype(np.float64).reshape(-1, torch.cuda.get_device_properties(
        eng.device).multi_processor_count, words)
    t0 = t[t > 0].min()
    t = np.where(t > 0, (t - t0) / 1000.0, np.nan)
    out, prev_end = [], None
    nk = t.shape[0]
    for k in range(nk - 2):
        layer, kind = (k // 4, KERNELS[k % 4]) if k < nk - 3 else (-1, "lm_head")
        start, wait, pro, loop, epi = (t[k, :, j] for j in range(5))
        issue, ready = t[k, :, 8:32], t[k, :, 32:56]
        lat = ready - issue
        row = {"k": k, "layer": layer, "kind": kind,
               "start_min": np.nanmin(start), "start_max": np.nanmax(start),
               "wait_ret_max": np.nanmax(wait), "prologue_med": np.nanmedian(pro - wait),
               "stream_med": np.nanmedian(loop - pro), "stream_max": np.nanmax(loop - pro),
               "epilogue_med": np.nanmedian(epi - loop), "end_max": np.nanmax(epi),
               "unit_latency_med": np.nanmedian(lat), "ready_gap_med": np.nanmedian(np.diff(ready, axis=1)),
               "x_loaded_med": np.nanmedian(t[k, :, 5] - wait), "reduced_med": np.nanmedian(t[k, :, 6] - wait),
               "gap_from_prev_end": None if prev_end is None else np.nanmin(start) - prev_end}
        prev_end = np.nanmax(epi)
        if layer in layers_shown or layer == -1:
            out.append({key: (round(float(v), 2) if v is not None else None) if not isinstance(v, str) else v
                        for key, v in row.items()})
    gemv_k = nk - 2                                          # the last two slots are attention kernels
    total = float(np.nanmax(t[gemv_k - 1, :, 4]) - np.nanmin(t[0, :, 0]))
    attn = []
    for k in (gemv_k, gemv_k + 1):
        row = t[k]
        if np.isnan(row[:, 0]).all():
            continue
        attn.append({"slot": "layer 0" if k == gemv_k else "middle layer",
                     "start": round(float(np.nanmin(row[:, 0])), 2), "wait_ret": round(float(np.nanmax(row[:, 1])), 2),
                     "positions_done": round(float(np.nanmax(row[:, 2])), 2),
                     "partial_done": round(float(np.nanmax(row[:, 3])), 2),
                     "cluster_sync": round(float(np.nanmax(row[:, 4])), 2),
                     "merged": round(float(np.nanmax(row[:, 5])), 2),
                     "staged_max": round(float(np.nanmax(row[:, 6])), 2),
                     "scores_max": round(float(np.nanmax(row[:, 7])), 2),
                     "softmax_max": round(float(np.nanmax(row[:, 8])), 2)})
    return {"step_span_us": round(total, 1), "kernels": out, "attention": attn}


def tree_of(n: int, vocab: int, seed: int = 0, widths=(4, 2)):
    """A draft tree of n nodes in breadth-first order (tokens, parents): every node of level d gets
    widths[d] children (1 past the listed levels) until there are n nodes."""
    import random
    rng = random.Random(seed)
    tokens, parents, level, d = [], [], [-1], 0
    while len(tokens) < n:
        w = widths[d] if d < len(widths) else 1
        nxt = []
        for par in level:
            for _ in range(w):
                if len(tokens) < n:
                    tokens.append(rng.randrange(vocab))
                    parents.append(par)
                    nxt.append(len(tokens) - 1)
        level, d = nxt, d + 1
    return tokens, parents


def sampling_steps(eng, nodes: int, repeat: int, top_k: int = 50, top_p: float = 0.9, temperature: float = 0.8) -> dict:
    """The device sampling path of one stochastic speculative round at the model's vocabulary, on
    seeded random logits: the top-k / top-p filter of the root row (`sp_sample_filter`) and the
    stochastic acceptance of a `nodes`-node tree (`sp_accept_stochastic`, target and drafter logits
    [nodes + 1, V]). Device milliseconds per round over `repeat` rounds (CUDA events), then one
    more round between cudaProfilerStart / Stop."""
    from .speculative import FlatForest, accept_stochastic, sample_filter
    V = eng.cfg.vocab
    g = torch.Generator(device=eng.device).manual_seed(0)
    tl = torch.randn((nodes + 1, V), generator=g, device=eng.device) * 3.0
    dl = tl + 0.5 * torch.randn((nodes + 1, V), generator=g, device=eng.device)
    tokens, parents = tree_of(nodes, V)
    # the tree as FlatForest fields: each root-to-leaf path as node ids and as tokens
    depths, chains = [], []
    for i, par in enumerate(parents):
        depths.append(1 if par < 0 else depths[par] + 1)
        chains.append((chains[par] if par >= 0 else ()) + (i,))
    leaves = [i for i in range(nodes) if i not in set(parents)]
    flat = FlatForest(tuple(tokens), tuple(parents), tuple(depths), tuple(chains[i] for i in leaves),
                      tuple(tuple(tokens[j] for j in chains[i]) for i in leaves))
    z = torch.empty((1, V), dtype=torch.float32, device=eng.device)

    def round_(counter):
        sample_filter(tl[0], temperature, top_k, top_p, out=z)
        return accept_stochastic(eng, flat, tl, dl, temperature, seed=7, counter=counter)

    first = round_(0)
    torch.cuda.synchronize()
    ms = None
    if repeat:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(repeat):
            round_(1 + i)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / repeat
    torch.cuda.cudart().cudaProfilerStart()
    round_(repeat + 1)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    eng.status()
    return {"vocab": V, "nodes": nodes, "top_k": top_k, "top_p": top_p, "temperature": temperature,
            "ms_per_round": ms, "first_round_emitted": list(first[0].emitted)}


def batch_steps(eng, B: int, repeat: int) -> dict:
    """B requests (the burst's prompt lengths) prefilled together, then batched decode steps: device
    milliseconds per step over `repeat` steps, then one more inside the profiler range."""
    from .randinit import burst_prompts
    prompts = burst_prompts(eng.cfg.vocab, B, 32, 128, seed=0)
    kvs = [eng.new_kv(len(p) + repeat + 8) for p in prompts]
    first = eng.prefill_batch(kvs, prompts).cpu().tolist()
    pos = [len(p) for p in prompts]
    out = eng.decode_batch(kvs, first, pos, 2)               # captures the step's graph
    toks, pos = out[-1].cpu().tolist(), [q + 2 for q in pos]
    torch.cuda.synchronize()
    ms = None
    if repeat:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = eng.decode_batch(kvs, toks, pos, repeat)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / repeat
        toks, pos = out[-1].cpu().tolist(), [q + repeat for q in pos]
    torch.cuda.cudart().cudaProfilerStart()
    out = eng.decode_batch(kvs, toks, pos, 1)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    eng.status()
    for kv in kvs:
        kv.close()
    res = {"model": eng.cfg.name, "requests": B, "decode_step_ms": ms, "tokens": out[-1].cpu().tolist()}
    eng.close()
    return res


def prompt_passes(eng, prompt, repeat: int, capacity: int) -> dict:
    """Prompt passes (device milliseconds per pass over `repeat` passes), then one more inside the
    profiler range."""
    kv = eng.new_kv(max(capacity, len(prompt)))
    for _ in range(2):
        kv.length = 0
        eng.forward(kv, prompt, want_logits=False, last_only=True)
    torch.cuda.synchronize()
    ms = None
    if repeat:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(repeat):
            kv.length = 0
            eng.forward(kv, prompt, want_logits=False, last_only=True)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / repeat
    kv.length = 0
    torch.cuda.cudart().cudaProfilerStart()
    _, am = eng.forward(kv, prompt, want_logits=False, last_only=True)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    eng.status()
    out = {"model": eng.cfg.name, "prompt": len(prompt), "prompt_pass_ms": ms, "argmax": int(am[-1])}
    eng.close()
    return out


def verify_passes(eng, prompt, nodes: int, repeat: int, capacity: int) -> dict:
    """Batched verify passes over an n-node tree after the prompt: device microseconds per pass
    (CUDA events over `repeat` graph replays), then one more pass inside the profiler range."""
    tokens, parents = tree_of(nodes, eng.cfg.vocab)
    kv = eng.new_kv(capacity)
    eng.forward(kv, prompt, want_logits=False, last_only=True)
    for _ in range(3):
        am, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
    torch.cuda.synchronize()
    us = None
    if repeat:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(repeat):
            eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000.0 / repeat
    torch.cuda.cudart().cudaProfilerStart()
    am, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    eng.status()
    out = {"model": eng.cfg.name, "prompt": len(prompt), "nodes": nodes, "verify_us": us, "argmax": am.cpu().tolist()}
    eng.close()
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="qwen2-1.5b", choices=sorted(PRESETS))
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--repeat", type=int, default=5, help="timed repetitions per mode (0: just run once)")
    ap.add_argument("--modes", default="graph+pdl")
    ap.add_argument("--capacity", type=int, default=4096)
    ap.add_argument("--prefetch-mb", default="0", help="comma list of L2 prefetch distances (MB) to compare")
    ap.add_argument("--evict-first", default="1", help="comma list of 0/1: stream weights with evict-first")
    ap.add_argument("--trace", action="store_true", help="print the kernel timeline of the last decode step")
    ap.add_argument("--step", default="step", help="comma list of step implementations: step (persistent), chain")
    ap.add_argument("--l2-kb", default="0", help="comma list: KB per CTA the step kernel warms L2 with ahead of its ring")
    ap.add_argument("--int8", action="store_true", help="blockwise-int8 random weights (drawn on the device)")
    ap.add_argument("--verify", type=int, default=0,
                    help="instead of decoding: after the prompt, `--repeat` + 1 batched verify passes of a tree of this "
                         "many nodes (branching 4, 2, 1, 1, ... breadth first); the last pass runs between "
                         "cudaProfilerStart / Stop (for ncu --profile-from-start off)")
    ap.add_argument("--prefill-pass", action="store_true",
                    help="instead of decoding: `--repeat` + 1 prompt passes of `--prompt` tokens (the batched pass, "
                         "last token's head only); the last runs between cudaProfilerStart / Stop")
    ap.add_argument("--batch", type=int, default=0,
                    help="instead of decoding one request: this many requests (prompts of 32..128 tokens, packed "
                         "into batched passes), then `--repeat` batched decode steps (sp_decode_batch) and one more "
                         "between cudaProfilerStart / Stop")
    ap.add_argument("--sampling", type=int, default=0,
                    help="instead of decoding: the device sampling path of a stochastic speculative round with a tree "
                         "of this many nodes at the model's vocabulary (seeded random logits): `--repeat` rounds "
                         "timed, one more between cudaProfilerStart / Stop")
    a = ap.parse_args()
    from .engine import CudaQwen2
    cfg = PRESETS[a.model]
    if a.int8:
        w = make_int8_blockwise(cfg, seed=0, device="cuda")
    else:
        w = make_weights(cfg, seed=0, dtype=torch.float16)
    fmt = "i8" if a.int8 else "f16"
    prompt = random_prompt(cfg.vocab, a.prompt, seed=0)
    if a.sampling:
        tiny = PRESETS["tiny-hd64"]
        eng = CudaQwen2(replace(tiny, vocab=cfg.vocab), make_weights(replace(tiny, vocab=cfg.vocab), seed=0, dtype=torch.float16))
        print(json.dumps(sampling_steps(eng, a.sampling, a.repeat)))
        return
    if a.verify:
        print(json.dumps(verify_passes(CudaQwen2(cfg, w, weight_format=fmt), prompt, a.verify, a.repeat, a.capacity)))
        return
    if a.batch:
        print(json.dumps(batch_steps(CudaQwen2(cfg, w, weight_format=fmt), a.batch, a.repeat)))
        return
    if a.prefill_pass:
        print(json.dumps(prompt_passes(CudaQwen2(cfg, w, weight_format=fmt), prompt, a.repeat, a.capacity)))
        return
    results = {}
    variants = [(m, pf, ev, sk, la) for sk in a.step.split(",") for m in a.modes.split(",")
                for pf in a.prefetch_mb.split(",") for ev in a.evict_first.split(",") for la in a.l2_kb.split(",")]
    for mode, pf, ev, sk, la in variants:
        graph, pdl = MODES[mode]
        os.environ["SEEDPLANE_GRAPH"], os.environ["SEEDPLANE_PDL"] = graph, pdl
        os.environ["SEEDPLANE_STEP"] = sk
        os.environ["SEEDPLANE_STEP_L2_KB"] = la
        os.environ["SEEDPLANE_L2_PREFETCH_MB"], os.environ["SEEDPLANE_EVICT_FIRST"] = pf, ev
        os.environ["SEEDPLANE_TRACE"] = "1" if a.trace else "0"
        label = f"{sk} {mode} l2_kb={la} evict_first={ev}" if sk == "step" else f"{sk} {mode} prefetch={pf}MB evict_first={ev}"
        eng = CudaQwen2(cfg, w, weight_format=fmt)
        kv = eng.new_kv(a.capacity)
        _, am = eng.forward(kv, prompt, want_logits=False)
        first = int(am[-1])
        out = torch.empty(a.tokens, dtype=torch.int32, device=eng.device)
        kv.length = a.prompt
        eng.decode(kv, first, a.prompt, a.tokens, out=out)
        torch.cuda.synchronize()
        eng.status()
        ref = out.cpu().tolist()
        if a.repeat:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            host = 0.0
            s.record()
            for _ in range(a.repeat):
                kv.length = a.prompt
                t0 = time.perf_counter()
                eng.decode(kv, first, a.prompt, a.tokens, out=out)
                host += time.perf_counter() - t0
            e.record()
            torch.cuda.synchronize()
            n = a.repeat * a.tokens
            results[label] = {"device_ms_per_token": s.elapsed_time(e) / n, "host_enqueue_ms_per_token": 1000 * host / n,
                             "tokens_equal": out.cpu().tolist() == ref}
        if a.trace:
            results[label + " trace"] = trace_summary(eng)
        eng.close()
        del eng, kv
        torch.cuda.empty_cache()
    print(json.dumps({"model": a.model, "weights": fmt, "prompt": a.prompt, "tokens": a.tokens, "results": results}))


if __name__ == "__main__":
    main()
