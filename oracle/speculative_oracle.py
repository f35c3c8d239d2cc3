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
* `accept_stochastic` -- stochastic tree acceptance (recursive rejection sampling at a
                      temperature, seeded counter RNG). The reference has NO stochastic verifier:
                      this restates the repository's own written rule, fp64 operation by
                      operation (own exp, fixed summation orders, splitmix64), so the GPU kernel's
                      decisions can be checked bit for bit. Parity unpinned against the reference.
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


# ---- stochastic tree acceptance (restatement of the GPU rule, bit for bit) ---------------------
_M64 = (1 << 64) - 1
_LN2_HI, _LN2_LO, _INV_LN2 = 6.93147180369123816490e-01, 1.90821492927058770002e-10, 1.44269504088896338700e+00
_INV_FACT = [1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0, 1.0 / 40320.0, 1.0 / 5040.0,
             1.0 / 720.0, 1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0, 0.5, 1.0, 1.0]
_THREADS = 256


def dexp_ref(x):
    """exp in fp64: Cody-Waite reduction by a two-part ln 2, Taylor series to r^13/13! in Horner
    form (no fused multiply-add), scaling by 2^k; 0 below -745."""
    import numpy as np
    x = np.asarray(x, dtype=np.float64)
    k = np.rint(x * _INV_LN2)
    r = (x + (-(k * _LN2_HI))) + (-(k * _LN2_LO))
    pw = np.full_like(x, 1.0 / 6227020800.0)
    for c in _INV_FACT:
        pw = pw * r + c
    with np.errstate(over="ignore"):
        out = np.ldexp(pw, np.where(x < -745.0, 0, k).astype(np.int64))
    return np.where(x < -745.0, 0.0, out)


def _block_sums(vals):
    """Contiguous blocks of ceil(V / 256) entries, each summed in index order, then the block sums
    in order: (block sums [256], total)."""
    import numpy as np
    V = vals.shape[0]
    B = -(-V // _THREADS)
    pad = np.zeros(_THREADS * B, dtype=np.float64)
    pad[:V] = vals
    blocks = pad.reshape(_THREADS, B)
    acc = np.zeros(_THREADS, dtype=np.float64)
    for i in range(B):
        acc = acc + blocks[:, i]
    tot = 0.0
    for t in range(_THREADS):
        tot = tot + float(acc[t])
    return acc, tot


def _splitmix(state):
    state = (state + 0x9E3779B97F4A7C15) & _M64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return state, z ^ (z >> 31)


def accept_stochastic(tokens, parents, target_logits, draft_logits, temperature: float, seed: int, counter: int):
    """The stochastic tree acceptance (see the GPU kernel's description): returns (emitted tokens,
    accepted node indices). `target_logits` / `draft_logits`: fp32 [n + 1, V], row 0 after the
    committed prefix, row i + 1 after node i."""
    import numpy as np
    tl = np.asarray(target_logits, dtype=np.float32).astype(np.float64)
    dl = np.asarray(draft_logits, dtype=np.float32).astype(np.float64)
    n, V = len(tokens), tl.shape[1]
    inv_t = 1.0 / float(temperature)
    state = (seed ^ ((counter * 0x9E3779B97F4A7C15) & _M64)) & _M64
    cur, emitted, accepted = -1, [], []
    for _ in range(n + 1):
        zt, zd = tl[cur + 1] * inv_t, dl[cur + 1] * inv_t
        mt, md = float(np.max(zt)), float(np.max(zd))
        et, ed = dexp_ref(zt + (-mt)), dexp_ref(zd + (-md))
        _, St = _block_sums(et)
        _, Sd = _block_sums(ed)
        P = et / St
        qv = ed / Sd
        nxt = -1
        for c in range(n):
            if parents[c] != cur:
                continue
            x = tokens[c]
            state, z = _splitmix(state)
            u = float(z >> 11) * 2.0 ** -53
            if u < float(P[x]) / float(qv[x]):
                nxt = c
                break
            res = np.fmax(P + (-qv), 0.0)
            _, Z = _block_sums(res)
            if Z > 0.0:
                P = res / Z
        if nxt >= 0:
            emitted.append(int(tokens[nxt]))
            accepted.append(nxt)
            cur = nxt
            if all(p != cur for p in parents):
                break
            continue
        state, z = _splitmix(state)
        u = float(z >> 11) * 2.0 ** -53
        blocks, S = _block_sums(P)
        target = u * S
        B = -(-V // _THREADS)
        run, pick, found = 0.0, V - 1, False
        for t in range(_THREADS):
            if found:
                break
            if run + float(blocks[t]) > target or t == _THREADS - 1:
                for i in range(B):
                    j = t * B + i
                    if j >= V:
                        break
                    run = run + float(P[j])
                    if run > target:
                        pick, found = j, True
                        break
                if not found:                      # rounding: the last positive index up to the block's end
                    j = min(V - 1, t * B + B - 1)
                    while j > 0 and not float(P[j]) > 0.0:
                        j -= 1
                    pick, found = (j if float(P[j]) > 0.0 else min(V - 1, t * B + B - 1)), True
            else:
                run = run + float(blocks[t])
        emitted.append(int(pick))
        break
    return emitted, accepted


# ---- top-k / top-p filter (restatement of the reference's sample(), qwen_engine.py:147-156) ------
def sample_filter(logits, temperature: float, top_k: int = 0, top_p: float = 1.0):
    """The reference's masking before its multinomial draw, in fp32 as torch computes it:
    z = logits / T; top_k > 0: -inf where z < the top_k-th largest z; top_p < 1: sort descending
    (stable), probs = softmax in fp32, -inf where cumsum(probs) - probs > top_p. Returns z (fp32)."""
    import numpy as np
    z = (np.asarray(logits, dtype=np.float32) / np.float32(temperature)).astype(np.float32)
    V = z.shape[0]
    if top_k > 0:
        cutoff = np.partition(z, V - min(top_k, V))[V - min(top_k, V)]
        z = np.where(z < cutoff, np.float32(-np.inf), z).astype(np.float32)
    if top_p < 1:
        order = np.argsort(-z, kind="stable")
        values = z[order]
        e = np.exp(values - values[0], dtype=np.float32)
        probs = (e / e.sum(dtype=np.float32)).astype(np.float32)
        drop = (np.cumsum(probs, dtype=np.float32) - probs) > np.float32(top_p)
        values = np.where(drop, np.float32(-np.inf), values).astype(np.float32)
        z = np.full_like(z, -np.inf)
        z[order] = values
    return z


def sample_filter_margin(logits, temperature: float, top_k: int = 0, top_p: float = 1.0) -> float:
    """How far the top-p decision is from flipping: min |exclusive mass - top_p| over the entries
    kept by top-k, in fp64 (inf when top_p >= 1). Cases with a margin below fp32 rounding are
    ambiguous between implementations that sum in different orders."""
    import numpy as np
    if top_p >= 1:
        return float("inf")
    z = sample_filter(logits, temperature, top_k, 1.0).astype(np.float64)
    v = np.sort(z[np.isfinite(z)])[::-1]
    e = np.exp(v - v[0])
    excl = (np.cumsum(e) - e) / e.sum()
    # the first entry's exclusive mass is exactly 0 everywhere: it never flips
    return float(np.min(np.abs(excl[1:] - top_p))) if excl.size > 1 else float("inf")
