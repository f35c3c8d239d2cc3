"""The product's `speculative` surface (CPU): identical types and decisions as the reference.

Checked against the golden decisions the reference's own `verify_greedy` produced
(`tests/golden/speculative.json`), against the reference's known-answer tests
(`tests/test_speculative.py:7-44`, restated), and `accept_greedy` (the batched rule on per-node
argmaxes) against the sequential rule."""
import hashlib
import json

import pytest

from seedplane_b200.speculative import (CommitLedger, SpeculativeForest, Verification, accept_greedy,
                                        verify_greedy)


def _hashed_target(prefix, vocab=8):
    h = hashlib.sha256(json.dumps(list(prefix)).encode()).digest()
    return [float(b % 5) for b in h[:vocab]]


def _predictions(committed, flat, target):
    full = {}
    for p, ids in zip(flat.paths, flat.node_paths):
        for d, nid in enumerate(ids):
            full[nid] = tuple(committed) + p[:d + 1]
    first = lambda v: max(range(len(v)), key=v.__getitem__)
    return first(target(tuple(committed))), [first(target(full[i])) for i in range(len(flat.tokens))]


def test_golden_decisions_sequential_and_batched(golden_dir):
    cases = json.loads((golden_dir / "speculative.json").read_text())["hashed_target"]
    for c in cases:
        forest = SpeculativeForest.build(c["branches"])
        assert forest.node_count == c["node_count"]
        want = Verification(tuple(c["emitted"]), c["accepted"], c["rejected"], c["steps"], tuple(c["branch"]))
        assert verify_greedy(c["committed"], forest, _hashed_target) == want
        flat = forest.flatten()
        root, preds = _predictions(c["committed"], flat, _hashed_target)
        got, nodes = accept_greedy(flat, root, preds)
        assert got == want
        # the accepted nodes are the chosen path's prefix of accepted draft tokens
        path_nodes = flat.node_paths[flat.paths.index(want.branch)] if want.branch else ()
        assert nodes == tuple(path_nodes[:want.accepted_draft_tokens])


def _kat_target(prefix):
    logits = [0.0] * 8
    logits[min(len(prefix), 5)] = 1.0
    return logits


def test_reference_known_answers():
    f = SpeculativeForest.build([[1, 2, 3], [1, 2, 4], [1, 5]])
    assert f.node_count == 5 and len(f.paths) == 3
    r = verify_greedy([0], SpeculativeForest.build([[1, 2, 7], [1, 2, 3, 4]]), _kat_target)
    assert r.branch == (1, 2, 3, 4) and r.emitted == (1, 2, 3, 4) and r.accepted_draft_tokens == 4 and not r.rejected
    r = verify_greedy([0], SpeculativeForest.build([[1, 2, 7]]), _kat_target)
    assert r.emitted == (1, 2, 3) and r.accepted_draft_tokens == 2 and r.rejected
    ledger = CommitLedger([0])
    r = verify_greedy(ledger.tokens, SpeculativeForest.build([[1, 2]]), _kat_target)
    assert ledger.frontier == 1
    ledger.commit(r)
    assert ledger.tokens == [0, 1, 2] and ledger.frontier == 3 and ledger.commits == 1
    r = verify_greedy([0], SpeculativeForest.build([]), _kat_target)
    assert r.emitted == (1,) and r.target_steps == 1
    with pytest.raises(ValueError):
        CommitLedger().commit(Verification((), 0, False, 0, ()))


def test_flatten_is_ancestor_closed_and_skips_empty_branches():
    flat = SpeculativeForest.build([(1, 2, 3), (), (1, 2, 4), (1, 5), (6,)]).flatten()
    assert flat.tokens == (1, 2, 3, 4, 5, 6)
    assert flat.parents == (-1, 0, 1, 1, 0, -1)
    assert flat.depths == (1, 2, 3, 3, 2, 1)
    assert flat.node_paths == ((0, 1, 2), (0, 1, 3), (0, 4), (5,))
    assert all(p < i for i, p in enumerate(flat.parents))
