"""Generate golden vectors of shard-window attention by running SeedPlane's own reference code.

    python tests/golden/make_window_golden.py --reference <path to the SeedPlane source tree>

Imports `seedplane.engine.ShardPlan` and `seedplane.qwen_engine.Qwen2Engine` from the given source
tree and applies the window definition the reference's own oracle uses
(`experiments/v19/oracle_windows.py:22-33`): position i's logits come from a fresh cache over
exactly the token indices of its ShardPlan window up to i, with original position ids; from the
last prompt position on, the argmax is the next token. Models are this repository's seeded
random-init checkpoints written as HF directories the reference loads unmodified.

Writes `tests/golden/windows.json`: per case the model, weight precision, K/V precision, plan,
prompt, greedy tokens and the window sizes at a few positions. Tests read the file; the
reference is needed only to make it. Run on a CPU box.
"""
from __future__ import annotations

import argparse
import json
import sys
import tempfile
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))

from seedplane_b200.config import PRESETS, QWEN2_0_5B  # noqa: E402
from seedplane_b200.randinit import TEST_INIT, checksum, make_weights, random_prompt  # noqa: E402
from make_golden import fp16_kv_cache, write_hf  # noqa: E402

# (model, weights dtype, fp16 K/V, prompt length, new tokens, (shard, halo, sinks) plans)
CASES = [
    ("tiny-hd64", "fp32", False, 12, 60, [(16, 8, 4), (16, 0, 0), (20, 12, 2), (8, 8, 6), (10, 4, 9)]),
    ("tiny-hd64", "fp16", True, 12, 60, [(16, 8, 4), (12, 6, 3)]),
    ("tiny-hd128", "fp16", True, 12, 60, [(16, 8, 4), (24, 4, 1)]),
    ("qwen2-0.5b", "fp16", False, 64, 40, [(32, 16, 4)]),
]


def run_case(ShardPlan, Qwen2Engine, model, wdtype, kv16, n_prompt, n_new, plans):
    cfg = PRESETS[model] if model in PRESETS else QWEN2_0_5B
    init = TEST_INIT if model.startswith("tiny") else {}
    dtype = torch.float16 if wdtype == "fp16" else torch.float32
    w = make_weights(cfg, seed=0, dtype=dtype, **init)
    prompt = random_prompt(cfg.vocab, n_prompt, seed=0)
    out = []
    with tempfile.TemporaryDirectory() as d:
        write_hf(Path(d), cfg, w)
        e = Qwen2Engine(d, "cpu")
        for shard, halo, sinks in plans:
            t0 = time.perf_counter()
            plan = ShardPlan(shard, halo, sinks)
            seq = list(prompt)
            total = n_prompt + n_new
            visible = {}
            for c0, c1, idx in plan.windows(total):
                for i in range(c0, c1):
                    visible[i] = [int(j) for j in idx[:len(idx) - (c1 - 1 - i)]]
            for i in range(total):
                if i + 1 < n_prompt:
                    continue                    # only positions whose argmax is a generated token
                idx = visible[i]
                cache = fp16_kv_cache(e, len(idx)) if kv16 else e.new_cache(len(idx))
                logits, _ = e.forward([seq[j] for j in idx], cache, positions=idx)
                if len(seq) < total:
                    seq.append(int(logits[-1].argmax()))
            sizes = {str(i): len(visible[i]) for i in sorted({n_prompt - 1, shard, shard + 1, total - 1})}
            out.append({"model": model, "weights": wdtype, "kv_fp16": kv16, "init": init,
                        "plan": {"shard": shard, "halo": halo, "sinks": sinks}, "prompt": prompt,
                        "tokens": seq[n_prompt:], "window_sizes": sizes, "weights_sha256": checksum(w)})
            print(model, wdtype, "kv16" if kv16 else "kv32", (shard, halo, sinks), seq[n_prompt:n_prompt + 8],
                  f"{time.perf_counter() - t0:.1f}s")
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="root of the SeedPlane source tree")
    ap.add_argument("--out", default=str(HERE))
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from seedplane.engine import ShardPlan
    from seedplane.qwen_engine import Qwen2Engine
    torch.set_num_threads(8)
    cases = []
    for case in CASES:
        cases += run_case(ShardPlan, Qwen2Engine, *case)
    (Path(a.out) / "windows.json").write_text(json.dumps({"torch": torch.__version__, "cases": cases}, indent=0))


if __name__ == "__main__":
    main()
