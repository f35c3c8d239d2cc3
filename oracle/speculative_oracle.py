"""CPU ORACLE for speculative verification — TEST INFRASTRUCTURE ONLY.

Restates SeedPlane's correctness prototype `seedplane/speculative.py` so the batched GPU tree
verifier can be checked decision by decision:

* `build_forest`   -- trie of draft branches, empty branches skipped, `paths` in input order,
                      node count = trie nodes                      (speculative.py:23-43)
* `verify_greedy`  -- every path walked in input order, one target argmax (first max index) per
                      step, first mismatch emits the target token and rejects; ranking by
                      (accepted_draft_tokens, len(emitted)) with strict '>' so the earliest path
                      wins ties; no bonus token on full acceptance; empty forest -> one target
                      token                                          (speculative.py:55-92)
* `commit`         -- ledger frontier advances only on commit        (speculative.py:95-111)

Added for the batched verifier (no counterpart in the reference, checked against the above):

* `flatten_forest` -- the trie as arrays (token, parent, depth) in first-visit order of the input
                      paths, plus each path as a node-index list.
* `accept_from_predictions` -- the same decision as `verify_greedy`, computed from the target's
                      argmax after the committed prefix (`root_pred`) and after each node
                      (`node_pred`). With consistent logits it returns the identical Verification.

Pinned against: the reference's own known-answer tests (`tests/test_speculative.py:7-44`) and
golden outputs of the reference `verify_greedy` (`tests/golden/make_golden.py`).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Sequence, Tuple


def build_forest(branches) -> Tuple[Dict, List[Tuple[int, ...]]]:
    roots: Dict[int, Dict] = {}
    paths: List[Tuple[int, ...]] = []
    for branch in branches:
        path = tuple(int(t) for t in branch)
        if not path:
            continue
        paths.append(path)
        level = roots
        for t in path:
            level = level.setdefault(t, {})
    return roots, paths


def node_count(roots: Dict) -> int:
    return sum(1 + node_count(children) for children in roots.values())


def first_argmax(values: Sequence[float]) -> int:
    best, idx = None, -1
    for i, v in enumerate(values):
        if best is None or v > best:
            best, idx = v, i
    return idx


def verify_greedy(committed: Sequence[int], paths: Sequence[Tuple[int, ...]],
                  target_logits: Callable[[tuple], Sequence[float]]):
    """Returns (emitted, accepted_draft_tokens, rejected, target_steps, branch)."""
    base = tuple(int(t) for t in committed)
    if not paths:
        logits = target_logits(base)
        if len(logits) == 0:
            raise ValueError("target returned empty logits")
        return ((first_argmax(logits),), 0, False, 1, ())
    best = None
    for path in paths:
        emitted: List[int] = []
        steps = 0
        rejected = False
        for draft in path:
            logits = target_logits(base + tuple(emitted))
            if len(logits) == 0:
                raise ValueError("target returned empty logits")
            target = first_argmax(logits)
            steps += 1
            if draft != target:
                emitted.append(target)
                rejected = True
                break
            emitted.append(draft)
        result = (tuple(emitted), len(emitted) - int(rejected), rejected, steps, tuple(path))
        if best is None or (result[1], len(result[0])) > (best[1], len(best[0])):
            best = result
    return best


def flatten_forest(paths: Sequence[Tuple[int, ...]]):
    """Nodes in first-visit order: tokens, parents (-1 = child of the committed prefix), depths
    (1 = first draft token), and each path as a list of node indices."""
    index: Dict[Tuple[int, ...], int] = {}
    tokens: List[int] = []
    parents: List[int] = []
    depths: List[int] = []
    node_paths: List[List[int]] = []
    for path in paths:
        ids = []
        for d in range(1, len(path) + 1):
            key = path[:d]
            if key not in index:
                index[key] = len(tokens)
                tokens.append(path[d - 1])
                parents.append(index[path[:d - 1]] if d > 1 else -1)
                depths.append(d)
            ids.append(index[key])
        node_paths.append(ids)
    return tokens, parents, depths, node_paths


def accept_from_predictions(paths, node_paths, tokens, root_pred: int, node_pred: Sequence[int]):
    """`verify_greedy`'s decision from per-node target argmaxes."""
    if not paths:
        return ((int(root_pred),), 0, False, 1, ())
    best = None
    for path, ids in zip(paths, node_paths):
        emitted: List[int] = []
        steps = 0
        rejected = False
        prev = -1
        for nid in ids:
            target = root_pred if prev < 0 else node_pred[prev]
            steps += 1
            if tokens[nid] != target:
                emitted.append(int(target))
                rejected = True
                break
            emitted.append(tokens[nid])
            prev = nid
        result = (tuple(emitted), len(emitted) - int(rejected), rejected, steps, tuple(path))
        if best is None or (result[1], len(result[0])) > (best[1], len(best[0])):
            best = result
    return best


class Ledger:
    def __init__(self, tokens=()):
        self.tokens = list(tokens)
        self.commits = 0

    @property
    def frontier(self) -> int:
        return len(self.tokens)

    def commit(self, emitted: Sequence[int]):
        if not emitted:
            raise ValueError("cannot commit an empty verification")
        self.tokens.extend(emitted)
        self.commits += 1
        return tuple(emitted)
