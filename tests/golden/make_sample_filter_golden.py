"""Golden kept sets of the reference's top-k / top-p sampling, made by its own code.

    python tests/golden/make_sample_filter_golden.py --reference <path to the SeedPlane source tree>

Calls `seedplane.qwen_engine.Qwen2Engine.sample` (qwen_engine.py:146-156) on seeded logits rows and
records the probability vector it hands to `torch.multinomial` (replaced by a recorder for the
call): the entries with a nonzero probability are the kept set. Logits row of a case:
`np.random.default_rng(seed).standard_normal(V).astype(np.float32) * np.float32(scale)`. Cases
whose top-p decision lies within 1e-6 of flipping (oracle margin) are left out: implementations
that sum in different orders may disagree there. Writes `sample_filter.json` beside this file.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.speculative_oracle import sample_filter_margin  # noqa: E402

CASES = [  # (V, scale, temperature, top_k, top_p)
    (1000, 3.0, 1.0, 0, 0.9), (1000, 3.0, 0.7, 50, 1.0), (1000, 3.0, 1.3, 40, 0.8), (1000, 3.0, 1.0, 1, 1.0),
    (1000, 3.0, 1.0, 0, 0.0), (1000, 3.0, 2.0, 200, 0.95), (1000, 1.0, 1.0, 0, 0.5), (1000, 3.0, 0.5, 999, 0.3),
    (151936, 4.0, 1.0, 0, 0.9), (151936, 4.0, 0.8, 64, 0.95), (151936, 4.0, 1.0, 1000, 1.0), (151936, 4.0, 1.2, 0, 0.7),
]


def logits_row(seed: int, V: int, scale: float) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(V).astype(np.float32) * np.float32(scale)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from seedplane.qwen_engine import Qwen2Engine
    seen = {}

    def recorder(probs, num_samples, *args, **kwargs):
        seen["p"] = probs.detach().clone()
        return torch.zeros(num_samples, dtype=torch.long)

    out = []
    orig = torch.multinomial
    torch.multinomial = recorder
    try:
        for seed in range(3):
            for V, scale, T, k, p in CASES:
                l = logits_row(seed, V, scale)
                if sample_filter_margin(l, T, k, p) < 1e-6:
                    continue
                Qwen2Engine.sample(torch.from_numpy(l.copy()), T, k, p)
                kept = torch.nonzero(seen["p"] > 0).flatten().tolist()
                out.append({"seed": seed, "V": V, "scale": scale, "temperature": T, "top_k": k, "top_p": p,
                            "kept": kept})
    finally:
        torch.multinomial = orig
    (HERE / "sample_filter.json").write_text(json.dumps({"cases": out}, separators=(",", ":")))
    print(f"{len(out)} cases, kept sizes {[len(c['kept']) for c in out]}")


if __name__ == "__main__":
    main()
