"""The CPU oracle against golden vectors produced by SeedPlane's own reference code.

The fixtures come from `tests/golden/make_golden.py`, which ran the reference `Qwen2Engine`
(`seedplane/qwen_engine.py`) and `verify_greedy` (`seedplane/speculative.py`) on the same seeded
checkpoints. Passing here is what makes the oracle trustworthy as the checker of the CUDA path.
"""
import hashlib
import json

import numpy as np
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from oracle import speculative_oracle as so
from seedplane_b200.config import PRESETS, QWEN2_0_5B
from seedplane_b200.randinit import TEST_INIT, checksum, make_weights

torch.set_num_threads(min(8, torch.get_num_threads()))


def assert_logits_close(got, want, rel=1e-4):
    """fp32 reorderings differ by ~1e-5 of the logit range; allow 1e-4 of max |logit|."""
    want = np.asarray(want)
    np.testing.assert_allclose(np.asarray(got), want, rtol=0, atol=rel * float(np.abs(want).max()))


@pytest.mark.parametrize("name", ["tiny-hd64", "tiny-hd128", "tiny-untied"])
def test_tiny_models_match_reference(name, golden_dir):
    g = np.load(golden_dir / f"qwen_{name}.npz")
    cfg = PRESETS[name]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    assert checksum(w) == str(g["weights_sha256"]), "random-init generator changed"
    prompt = g["prompt"].tolist()
    o = OracleQwen2(cfg, w)
    logits, _ = o.forward(prompt, o.new_cache(64), all_logits=True)
    assert_logits_close(logits.numpy(), g["all_logits"])
    shifted, _ = o.forward(prompt, o.new_cache(64), all_logits=True, positions=[p + 40 for p in range(len(prompt))])
    assert_logits_close(shifted.numpy(), g["shifted_logits"])
    toks, _ = o.greedy(prompt, 8, capacity=64)
    assert toks == g["greedy"].tolist()
    cache = o.new_cache(64)
    _, cache = o.forward(prompt[:7], cache)
    chunk2, _ = o.forward(prompt[7:], cache, all_logits=True)
    assert_logits_close(chunk2.numpy(), g["chunk2_logits"])
    # fp16 K/V at cache write
    o16 = OracleQwen2(cfg, w, kv_fp16=True)
    logits16, _ = o16.forward(prompt, o16.new_cache(64), all_logits=True)
    assert_logits_close(logits16.numpy(), g["all_logits_kv16"])
    toks16, _ = o16.greedy(prompt, 8, capacity=64)
    assert toks16 == g["greedy_kv16"].tolist()


@pytest.mark.slow
@pytest.mark.parametrize("label,dtype", [("fp32", torch.float32), ("fp16_weights", torch.float16)])
def test_qwen2_0_5b_reference_config(label, dtype, golden_dir):
    """The reference's own CPU case: Qwen2-0.5B random-init, 64-token prompt, 32 greedy tokens."""
    gold = json.loads((golden_dir / "qwen2-0.5b.json").read_text())
    w = make_weights(QWEN2_0_5B, seed=0, dtype=dtype)
    o = OracleQwen2(QWEN2_0_5B, w)
    toks, margins = o.greedy(gold["prompt"], 32)
    assert toks == gold[label]["tokens"]
    assert hashlib.sha256(json.dumps(toks).encode()).hexdigest() == gold[label]["sha256"]
    np.testing.assert_allclose(margins, gold[label]["margins"], atol=2e-4)


def _hashed_target(prefix, vocab=8):
    h = hashlib.sha256(json.dumps(list(prefix)).encode()).digest()
    return [float(b % 5) for b in h[:vocab]]


def test_verify_greedy_matches_reference_on_random_forests(golden_dir):
    cases = json.loads((golden_dir / "speculative.json").read_text())["hashed_target"]
    assert len(cases) == 80
    for c in cases:
        roots, paths = so.build_forest(c["branches"])
        assert so.node_count(roots) == c["node_count"]
        got = so.verify_greedy(c["committed"], paths, _hashed_target)
        want = (tuple(c["emitted"]), c["accepted"], c["rejected"], c["steps"], tuple(c["branch"]))
        assert got == want, c
        # the batched decision from per-node predictions is identical
        toks, parents, depths, node_paths = so.flatten_forest(paths)
        full = {}
        for p, ids in zip(paths, node_paths):
            for d, nid in enumerate(ids):
                full[nid] = tuple(c["committed"]) + p[:d + 1]
        root_pred = so.first_argmax(_hashed_target(tuple(c["committed"])))
        node_pred = [so.first_argmax(_hashed_target(full[i])) for i in range(len(toks))]
        assert so.accept_from_predictions(paths, node_paths, toks, root_pred, node_pred) == want, c


def test_forest_flattening_is_ancestor_closed():
    toks, parents, depths, node_paths = so.flatten_forest([(1, 2, 3), (1, 2, 4), (1, 5), (6,)])
    assert toks == [1, 2, 3, 4, 5, 6]
    assert parents == [-1, 0, 1, 1, 0, -1]
    assert depths == [1, 2, 3, 3, 2, 1]
    assert node_paths == [[0, 1, 2], [0, 1, 3], [0, 4], [5]]
    for i, p in enumerate(parents):
        assert p < i


class _ReferenceKATs:
    """The reference's known-answer tests (`tests/test_speculative.py:7-44`), applied to the oracle."""

    @staticmethod
    def target(prefix):
        expected = min(len(prefix), 5)
        logits = [0.0] * 8
        logits[expected] = 1.0
        return logits


def test_reference_kats_on_oracle():
    t = _ReferenceKATs.target
    roots, paths = so.build_forest([[1, 2, 3], [1, 2, 4], [1, 5]])
    assert so.node_count(roots) == 5 and len(paths) == 3
    _, paths = so.build_forest([[1, 2, 7], [1, 2, 3, 4]])
    r = so.verify_greedy([0], paths, t)
    assert r[4] == (1, 2, 3, 4) and r[0] == (1, 2, 3, 4) and r[1] == 4 and not r[2]
    _, paths = so.build_forest([[1, 2, 7]])
    r = so.verify_greedy([0], paths, t)
    assert r[0] == (1, 2, 3) and r[1] == 2 and r[2]
    ledger = so.Ledger([0])
    _, paths = so.build_forest([[1, 2]])
    r = so.verify_greedy(ledger.tokens, paths, t)
    assert ledger.frontier == 1
    ledger.commit(r[0])
    assert ledger.tokens == [0, 1, 2] and ledger.frontier == 3 and ledger.commits == 1
    r = so.verify_greedy([0], [], t)
    assert r[0] == (1,) and r[3] == 1
