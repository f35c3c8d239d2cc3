"""Generate golden vectors by running SeedPlane's own reference code (not the oracle).

    python tests/golden/make_golden.py --reference <path to the SeedPlane source tree>

Imports `seedplane.qwen_engine.Qwen2Engine` and `seedplane.speculative` from the given source
tree, feeds them this repository's seeded random-init checkpoints (written as an HF directory the
reference loads unmodified), and stores what they return under `tests/golden/`:

* `qwen_<model>.npz`  -- tiny models (init `TEST_INIT`): all-row prefill logits, greedy tokens, position-shifted
                         logits, and the same with K/V rounded to fp16 at cache write.
* `qwen2-0.5b.json`   -- the reference's own CPU configuration (fp32, 64-token prompt, 32 greedy
                         tokens): tokens, per-step top-2 margins, top-8 logits of two steps; and the
                         same prompt with fp16-rounded weights.
* `speculative.json`  -- `verify_greedy` on random forests with a deterministic target, and on a
                         tiny model target.

The reference is needed only to *make* these files; tests read the files. Run on a CPU box.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import random
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from seedplane_b200.config import PRESETS, QWEN2_0_5B  # noqa: E402
from seedplane_b200.randinit import TEST_INIT, checksum, make_weights, random_prompt  # noqa: E402


def write_hf(directory: Path, cfg, weights):
    from safetensors.torch import save_file
    (directory / "config.json").write_text(json.dumps(cfg.to_hf()))
    save_file({k: v.float().contiguous() for k, v in weights.items()}, str(directory / "model.safetensors"))


class Fp16KV(torch.Tensor):
    """fp32 cache tensor that rounds whatever is copied into it to fp16 (K/V stored as fp16)."""

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is torch.Tensor.copy_:
            args = (args[0], args[1].half().float()) + tuple(args[2:])
        return super().__torch_function__(func, types, args, kwargs)


def fp16_kv_cache(engine, capacity):
    cache = engine.new_cache(capacity)
    cache.keys = [k.zero_().as_subclass(Fp16KV) for k in cache.keys]
    cache.values = [v.zero_().as_subclass(Fp16KV) for v in cache.values]
    return cache


def greedy(engine, prompt, n, cache):
    logits, cache = engine.forward(prompt, cache)
    toks, margins, tops = [], [], []
    for i in range(n):
        row = logits[-1].float()
        top = torch.topk(row, 8)
        toks.append(int(row.argmax()))
        margins.append(float(top.values[0] - top.values[1]))
        tops.append((top.values.tolist(), top.indices.tolist()))
        if i + 1 < n:
            logits, cache = engine.forward([toks[-1]], cache)
    return toks, margins, tops


def tiny_case(Qwen2Engine, name, out: Path):
    cfg = PRESETS[name]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    with tempfile.TemporaryDirectory() as d:
        write_hf(Path(d), cfg, w)
        e = Qwen2Engine(d, "cpu")
        all_logits, _ = e.forward(prompt, e.new_cache(64), all_logits=True)
        shifted, _ = e.forward(prompt, e.new_cache(64), all_logits=True,
                               positions=[p + 40 for p in range(len(prompt))])
        toks, margins, _ = greedy(e, prompt, 8, e.new_cache(64))
        all16, _ = e.forward(prompt, fp16_kv_cache(e, 64), all_logits=True)
        toks16, margins16, _ = greedy(e, prompt, 8, fp16_kv_cache(e, 64))
        # Decode-step logits after a 2-chunk prefill (exercises the start > 0 mask path).
        cache = e.new_cache(64)
        _, cache = e.forward(prompt[:7], cache)
        chunk2, cache = e.forward(prompt[7:], cache, all_logits=True)
    np.savez_compressed(out / f"qwen_{name}.npz", prompt=np.array(prompt, np.int64),
                        all_logits=all_logits.numpy(), shifted_logits=shifted.numpy(),
                        greedy=np.array(toks, np.int64), margins=np.array(margins),
                        all_logits_kv16=all16.numpy(), greedy_kv16=np.array(toks16, np.int64),
                        chunk2_logits=chunk2.numpy(), weights_sha256=np.array(checksum(w)))
    print(name, "greedy", toks, "kv16", toks16, "min margin", min(margins))


def cfg1_case(Qwen2Engine, out: Path):
    cfg = QWEN2_0_5B
    prompt = random_prompt(cfg.vocab, 64, seed=0)
    result = {"config": cfg.as_dict(), "prompt": prompt, "torch": torch.__version__}
    for label, dtype in (("fp32", torch.float32), ("fp16_weights", torch.float16)):
        w = make_weights(cfg, seed=0, dtype=dtype)
        with tempfile.TemporaryDirectory() as d:
            write_hf(Path(d), cfg, w)
            e = Qwen2Engine(d, "cpu")
            t0 = time.perf_counter()
            toks, margins, tops = greedy(e, prompt, 32, e.new_cache(len(prompt) + 32))
            dt = time.perf_counter() - t0
        result[label] = {"tokens": toks, "margins": margins, "top8_step0": tops[0], "top8_step31": tops[-1],
                         "sha256": hashlib.sha256(json.dumps(toks).encode()).hexdigest(),
                         "weights_sha256": checksum(w), "seconds": dt}
        print("qwen2-0.5b", label, toks[:8], "min margin", min(margins), f"{dt:.1f}s")
        del w
    (out / "qwen2-0.5b.json").write_text(json.dumps(result, indent=1))


def hashed_target(prefix, vocab=8):
    """Deterministic synthetic target: logits from a hash of the prefix, with occasional ties."""
    h = hashlib.sha256(json.dumps(list(prefix)).encode()).digest()
    return [float(b % 5) for b in h[:vocab]]


def speculative_cases(spec, Qwen2Engine, out: Path):
    rng = random.Random(0)
    cases = []
    for i in range(60):
        nb = rng.randint(0, 6)
        branches = [[rng.randint(0, 7) for _ in range(rng.randint(0, 5))] for _ in range(nb)]
        committed = [rng.randint(0, 7) for _ in range(rng.randint(0, 3))]
        forest = spec.SpeculativeForest.build(branches)
        v = spec.verify_greedy(committed, forest, hashed_target)
        cases.append({"committed": committed, "branches": branches, "node_count": forest.node_count,
                      "emitted": list(v.emitted), "accepted": v.accepted_draft_tokens, "rejected": v.rejected,
                      "steps": v.target_steps, "branch": list(v.branch)})
    # A "follow the target" family: drafts agree with the target for a while, then diverge.
    for i in range(20):
        committed = [rng.randint(0, 7) for _ in range(2)]
        branches = []
        for _ in range(rng.randint(1, 5)):
            path, prefix = [], tuple(committed)
            for d in range(rng.randint(1, 5)):
                logits = hashed_target(prefix)
                t = max(range(len(logits)), key=logits.__getitem__)
                if rng.random() < 0.25:
                    t = (t + rng.randint(1, 7)) % 8
                path.append(t)
                prefix = prefix + (t,)
            branches.append(path)
        forest = spec.SpeculativeForest.build(branches)
        v = spec.verify_greedy(committed, forest, hashed_target)
        cases.append({"committed": committed, "branches": branches, "node_count": forest.node_count,
                      "emitted": list(v.emitted), "accepted": v.accepted_draft_tokens, "rejected": v.rejected,
                      "steps": v.target_steps, "branch": list(v.branch)})

    # Model-driven: a tiny fp16-rounded target, prefix logits from a fresh forward per call.
    cfg = PRESETS["tiny-hd64"]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    model_cases = []
    with tempfile.TemporaryDirectory() as d:
        write_hf(Path(d), cfg, w)
        e = Qwen2Engine(d, "cpu")

        def target(prefix):
            logits, _ = e.forward(list(prefix), e.new_cache(len(prefix)))
            return logits[-1].tolist()

        for i in range(6):
            committed = random_prompt(cfg.vocab, 10, seed=50 + i)
            greedy_path, prefix = [], tuple(committed)
            for _ in range(4):
                row = target(prefix)
                t = max(range(len(row)), key=row.__getitem__)
                greedy_path.append(t)
                prefix += (t,)
            branches = [greedy_path[:2] + [(greedy_path[2] + 1) % cfg.vocab],
                        greedy_path[:4] if i % 2 == 0 else greedy_path[:3] + [(greedy_path[3] + 5) % cfg.vocab],
                        [(greedy_path[0] + 3) % cfg.vocab, 17],
                        greedy_path[:1]]
            forest = spec.SpeculativeForest.build(branches)
            v = spec.verify_greedy(committed, forest, target)
            model_cases.append({"committed": committed, "branches": branches, "node_count": forest.node_count,
                                "emitted": list(v.emitted), "accepted": v.accepted_draft_tokens,
                                "rejected": v.rejected, "steps": v.target_steps, "branch": list(v.branch)})
    (out / "speculative.json").write_text(json.dumps({"hashed_target": cases, "tiny_model": model_cases,
                                                      "tiny_model_config": "tiny-hd64"}, indent=0))
    print("speculative", len(cases), "hashed cases,", len(model_cases), "model cases")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="root of the SeedPlane source tree")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--skip-cfg1", action="store_true")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from seedplane.qwen_engine import Qwen2Engine
    from seedplane import speculative as spec
    torch.set_num_threads(8)
    out = Path(a.out)
    for name in ("tiny-hd64", "tiny-hd128", "tiny-untied"):
        tiny_case(Qwen2Engine, name, out)
    speculative_cases(spec, Qwen2Engine, out)
    if not a.skip_cfg1:
        cfg1_case(Qwen2Engine, out)


if __name__ == "__main__":
    main()
