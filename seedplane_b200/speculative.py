"""Speculative decoding surface of the B200 engine (drop-in for `seedplane.speculative`).

Same types and the same decisions as the reference prototype (`seedplane/speculative.py`):

* `SpeculativeForest.build` / `node_count` -- trie of draft branches, empty branches skipped,
  `paths` kept in input order (speculative.py:18-43).
* `verify_greedy(committed, forest, target_logits)` -- every path walked in input order; the
  target token is the first index of the maximum; the first mismatch emits the target token and
  rejects; the path with the largest (accepted_draft_tokens, len(emitted)) wins, the earliest on
  ties (strict '>'); no bonus token on full acceptance; an empty forest yields one target token
  (speculative.py:55-92).
* `CommitLedger` -- the committed frontier moves only on commit (speculative.py:95-111).

Added for the GPU:

* `SpeculativeForest.flatten()` -- the trie as arrays (token, parent, depth) in first-visit order
  of the paths, and each path as a list of node indices: the layout `sp_verify_tree` takes.
* `verify_tree(engine, kv, forest, root_pred, base_pos)` -- ONE batched target pass over the whole
  forest on the device (every node attends to the committed prefix and its own ancestors), then
  the same selection rule applied to the per-node argmaxes. Returns the same `Verification` as
  `verify_greedy` would with the engine's logits, plus the data needed to commit.
* `commit_tree(engine, kv, tree, verification)` -- moves the accepted nodes' K/V into place.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple


@dataclass
class ForestNode:
    token: int
    children: Dict[int, "ForestNode"] = field(default_factory=dict)


@dataclass
class SpeculativeForest:
    """Draft branches merged into a trie: `roots` maps a first token to its node, `paths` keeps every
    non-empty branch as given (input order decides ties between equally good branches)."""
    roots: Dict[int, ForestNode] = field(default_factory=dict)
    paths: List[Tuple[int, ...]] = field(default_factory=list)

    @classmethod
    def build(cls, branches: Iterable[Iterable[int]]) -> "SpeculativeForest":
        forest = cls()
        for branch in branches:
            forest.add(branch)
        return forest

    def add(self, branch: Iterable[int]) -> None:
        """Merge one branch into the trie (an empty branch adds nothing)."""
        path = tuple(map(int, branch))
        if not path:
            return
        self.paths.append(path)
        level = self.roots
        for tok in path:
            if tok not in level:
                level[tok] = ForestNode(tok)
            level = level[tok].children

    @property
    def node_count(self) -> int:
        n, todo = 0, list(self.roots.values())
        while todo:
            node = todo.pop()
            n += 1
            todo.extend(node.children.values())
        return n

    def flatten(self) -> "FlatForest":
        index: Dict[Tuple[int, ...], int] = {}
        tokens: List[int] = []
        parents: List[int] = []
        depths: List[int] = []
        node_paths: List[List[int]] = []
        for path in self.paths:
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
        return FlatForest(tuple(tokens), tuple(parents), tuple(depths), tuple(tuple(p) for p in node_paths),
                          tuple(self.paths))


@dataclass(frozen=True)
class FlatForest:
    tokens: Tuple[int, ...]          # node tokens, first-visit order
    parents: Tuple[int, ...]         # parent node index, -1 = child of the committed prefix
    depths: Tuple[int, ...]          # 1 = first draft token
    node_paths: Tuple[Tuple[int, ...], ...]
    paths: Tuple[Tuple[int, ...], ...]


@dataclass(frozen=True)
class Verification:
    emitted: Tuple[int, ...]
    accepted_draft_tokens: int
    rejected: bool
    target_steps: int
    branch: Tuple[int, ...]


def _first_argmax(values: Sequence[float]) -> int:
    """Index of the largest value, the lowest index on ties (like `max` over the indices)."""
    if not len(values):
        raise ValueError("target returned empty logits")
    best = 0
    for i in range(1, len(values)):
        if values[i] > values[best]:
            best = i
    return best


def _select(flat: FlatForest, predict: Callable[[int], int]) -> Tuple[Verification, Tuple[int, ...]]:
    """The greedy decision over a flattened forest. `predict(node)` is the target's token after
    node `node` (-1: after the committed prefix alone); it is asked only for the nodes a walk
    reaches, each at most once.

    Each path is walked from its root while the target agrees with the draft; the first
    disagreement emits the target's token instead and rejects the path; a fully agreed path
    emits its draft tokens and nothing more. The decision is the path with the most accepted
    draft tokens, then the most emitted tokens, then the earliest in input order. Returns it with
    the node indices of its accepted draft tokens."""
    if not flat.paths:
        return Verification((predict(-1),), 0, False, 1, ()), ()
    memo: Dict[int, int] = {}

    def after(node: int) -> int:
        if node not in memo:
            memo[node] = int(predict(node))
        return memo[node]

    best_key, best = None, None
    for order, (path, ids) in enumerate(zip(flat.paths, flat.node_paths)):
        emitted: List[int] = []
        prev = -1
        for nid in ids:
            want = after(prev)
            if want != flat.tokens[nid]:
                emitted.append(want)
                break
            emitted.append(flat.tokens[nid])
            prev = nid
        accepted = ids.index(prev) + 1 if prev >= 0 else 0
        rejected = len(emitted) > accepted
        key = (accepted, len(emitted), -order)
        if best_key is None or key > best_key:
            best_key = key
            best = (Verification(tuple(emitted), accepted, rejected, len(emitted), tuple(path)), tuple(ids[:accepted]))
    return best


def verify_greedy(committed: Sequence[int], forest: SpeculativeForest,
                  target_logits: Callable[[Tuple[int, ...]], Sequence[float]]) -> Verification:
    """The reference's greedy verification with a logits callback: `target_logits(prefix)` gives the
    target's logits for the token after `prefix`. Every distinct prefix is asked once (paths that
    share a trie prefix share its answers); the decision is `_select`'s. The GPU path is
    `verify_tree`."""
    base = tuple(int(t) for t in committed)
    flat = forest.flatten()
    prefix_of = {}
    for path, ids in zip(flat.paths, flat.node_paths):
        for d, nid in enumerate(ids):
            prefix_of[nid] = path[:d + 1]

    def predict(node: int) -> int:
        return _first_argmax(target_logits(base + (prefix_of[node] if node >= 0 else ())))

    return _select(flat, predict)[0]


def accept_greedy(flat: FlatForest, root_pred: int, node_pred: Sequence[int]) -> Tuple[Verification, Tuple[int, ...]]:
    """`verify_greedy`'s decision from the target argmax after the committed prefix (`root_pred`)
    and after each node (`node_pred[i]`). Returns the verification and the accepted draft nodes
    of the chosen path (their K/V is what a commit keeps)."""
    return _select(flat, lambda node: int(root_pred) if node < 0 else int(node_pred[node]))


def accept_greedy_device(engine, flat: FlatForest, root_pred: int, node_pred_dev
                         ) -> Tuple[Verification, Tuple[int, ...], Optional[int]]:
    """`accept_greedy` on the device (`sp_accept_greedy`): the same decision from the per-node
    argmaxes that stay in device memory (int32 [n] on the engine's device); only the decision comes
    back. Returns the verification, the accepted draft nodes and the target's token after a fully
    accepted path (None otherwise)."""
    import ctypes as C
    from . import _native as N
    from .engine import _stream
    n = len(flat.tokens)
    ends = [ids[-1] for ids in flat.node_paths]
    out = (C.c_int32 * (2 * n + 5))()
    ptr = C.c_void_p(node_pred_dev.data_ptr()) if n else C.c_void_p(None)
    N.check(N.load().sp_accept_greedy(engine.handle, ptr, int(root_pred), N.int_array(flat.tokens),
                                      N.int_array(flat.parents), n, N.int_array(ends), len(ends), out,
                                      C.c_void_p(_stream(engine.device))))
    n_out, n_acc, chosen, nxt = out[0], out[1], out[2], out[3]
    emitted = tuple(out[4 + i] for i in range(n_out))
    nodes = tuple(out[4 + n + 1 + i] for i in range(n_acc))
    path = tuple(flat.paths[chosen]) if chosen >= 0 else ()
    rejected = chosen >= 0 and n_out > n_acc          # no draft: the target's token, nothing rejected
    return Verification(emitted, n_acc, rejected, n_out, path), nodes, (nxt if nxt >= 0 else None)


@dataclass(frozen=True)
class TreeResult:
    verification: Verification
    accepted_nodes: Tuple[int, ...]  # node indices of the accepted draft tokens, in order
    node_pred: Optional[Tuple[int, ...]]   # target argmax after every node (None: decided on the device)
    next_pred: Optional[int]         # target argmax after the emitted tokens, when known (full acceptance)
    flat: FlatForest


def verify_tree(engine, kv, forest: SpeculativeForest, root_pred: int, base_pos: int,
                want_logits: bool = False, on_device: bool = True) -> TreeResult:
    """One batched target pass over the whole forest (`sp_verify_tree`) and the reference's
    selection rule on its argmaxes: on the device (`sp_accept_greedy`, only the decision is read
    back) or, with on_device=False, on the host over the argmaxes read back.

    `root_pred` is the target's greedy token after the committed prefix (the caller has it from
    the previous step); `base_pos` is the position of the first draft token. The cache length is
    not advanced; `commit_tree` keeps the accepted nodes."""
    flat = forest.flatten()
    if not flat.tokens:
        return TreeResult(Verification((int(root_pred),), 0, False, 1, ()), (), (), None, flat)
    argmax, _ = engine.verify_tree(kv, list(flat.tokens), list(flat.parents), base_pos, want_logits=want_logits)
    if on_device:
        ver, nodes, next_pred = accept_greedy_device(engine, flat, root_pred, argmax)
        return TreeResult(ver, nodes, None, next_pred, flat)
    node_pred = tuple(int(t) for t in argmax.cpu().tolist())
    ver, nodes = accept_greedy(flat, root_pred, node_pred)
    next_pred = node_pred[nodes[-1]] if (nodes and not ver.rejected) else None
    return TreeResult(ver, nodes, node_pred, next_pred, flat)


def accept_stochastic(engine, flat: FlatForest, target_logits, draft_logits, temperature: float, seed: int,
                      counter: int) -> Tuple[Verification, Tuple[int, ...]]:
    """Stochastic acceptance of a verified tree on the device (`sp_accept_stochastic`): children
    tried in node order with min(1, p/q), the residual max(p - q, 0) after each rejection, a draw
    from the residual when all are rejected; counter-based RNG, so (seed, counter) reproduce a
    decision. Logits fp32 [n + 1, V] on the engine's device: row 0 after the committed prefix, row
    i + 1 after node i. Returns the Verification and the accepted node indices."""
    import ctypes as C
    from . import _native as N
    from .engine import _stream
    n = len(flat.tokens)
    out = (C.c_int32 * (2 * n + 3))()
    N.check(N.load().sp_accept_stochastic(engine.handle, C.c_void_p(target_logits.data_ptr()),
                                          C.c_void_p(draft_logits.data_ptr()), target_logits.stride(0),
                                          target_logits.shape[1], N.int_array(flat.tokens), N.int_array(flat.parents),
                                          n, float(temperature), int(seed), int(counter), out,
                                          C.c_void_p(_stream(engine.device))))
    n_out, n_acc = out[0], out[1]
    emitted = tuple(out[2 + i] for i in range(n_out))
    nodes = tuple(out[2 + n + 1 + i] for i in range(n_acc))
    path = tuple(flat.tokens[i] for i in nodes)
    return Verification(emitted, n_acc, n_out > n_acc, n_out, path), nodes


def sample_filter(logits_row, temperature: float, top_k: int = 0, top_p: float = 1.0, out=None):
    """The masking of the reference's sample() (qwen_engine.py:147-156) on the device
    (`sp_sample_filter`): z = logits / temperature, -inf where top_k (> 0) or top_p (< 1) drops the
    entry. `logits_row`: fp32 [V] or [1, V] on a CUDA device; returns z fp32 [1, V]."""
    import ctypes as C
    import torch
    from . import _native as N
    from .engine import _stream
    row = logits_row.reshape(1, -1)
    if row.dtype != torch.float32 or not row.is_cuda or not row.is_contiguous():
        raise ValueError("logits_row must be a contiguous fp32 CUDA tensor")
    z = torch.empty_like(row) if out is None else out
    N.check(N.load().sp_sample_filter(C.c_void_p(row.data_ptr()), row.shape[1], float(temperature), int(top_k),
                                      float(top_p), C.c_void_p(z.data_ptr()), C.c_void_p(_stream(row.device))))
    return z


def sample_token(engine, logits_row, temperature: float, seed: int, counter: int, top_k: int = 0,
                 top_p: float = 1.0) -> int:
    """One draw from softmax(logits / temperature) on the device: the stochastic acceptance of an
    empty tree (`sp_accept_stochastic` with no nodes draws from the target distribution), with the
    same fp64 arithmetic and counter-based RNG, so (seed, counter) reproduce the token. With top_k
    (> 0) or top_p (< 1) the row first goes through `sample_filter` and the draw runs at temperature
    1 on its output. `logits_row`: fp32 [1, V] (or [V]) on the engine's device."""
    row = logits_row.reshape(1, -1)
    if top_k > 0 or top_p < 1.0:
        row = sample_filter(row, temperature, top_k, top_p)
        temperature = 1.0
    empty = FlatForest(tokens=(), parents=(), depths=(), node_paths=(), paths=())
    v, _ = accept_stochastic(engine, empty, row, row, temperature, seed, counter)
    return int(v.emitted[0])


def commit_tree(engine, kv, result: TreeResult) -> int:
    """Keep the K/V of the accepted draft nodes (they were written at scratch slots len + i) and
    advance the cache length by their number. Returns the new length."""
    base = kv.length
    slots = [base + i for i in result.accepted_nodes]
    engine.kv_commit(kv, slots)
    return kv.length


@dataclass
class CommitLedger:
    """The committed tokens. Only `commit` moves the frontier; speculation never touches it."""
    tokens: List[int] = field(default_factory=list)
    commits: int = 0

    @property
    def frontier(self) -> int:
        return len(self.tokens)

    def commit(self, verification: Verification) -> Tuple[int, ...]:
        new = tuple(verification.emitted)
        if len(new) == 0:
            raise ValueError("a verification that emitted no token cannot be committed")
        self.tokens += new
        self.commits += 1
        return new


# ---- tree drafting and the speculative decode loop (the cfg2 workload) ---------------------------
def draft_tree(drafter, dkv, root_logits, base_pos: int, branching=(4, 2, 1, 1), max_nodes: int = 16
               ) -> SpeculativeForest:
    """A draft tree from a drafter engine whose cache holds the committed prefix.

    Depth d expands every node of depth d - 1 into its drafter top-`branching[d-1]` children (one
    batched tree pass of the drafter per depth, `verify_tree` with logits, then `topk` on the
    device). The kept nodes are the `max_nodes` of highest cumulative drafter log-probability
    (ties: earlier node first), an ancestor-closed set because a child's cumulative log-probability
    never exceeds its parent's. Returned as a forest of root-to-leaf paths in node order; the
    drafter cache length is left unchanged (tree nodes sit at scratch slots)."""
    import torch
    tokens: List[int] = []
    parents: List[int] = []
    cum: List[float] = []
    idx, val, lse = drafter.topk(root_logits.reshape(1, -1).float().contiguous(), branching[0])
    frontier = []
    for t, v in zip(idx[0].tolist(), (val[0] - lse[0]).tolist()):
        tokens.append(int(t))
        parents.append(-1)
        cum.append(float(v))
        frontier.append(len(tokens) - 1)
    for width in branching[1:]:
        if not frontier or len(tokens) >= 4 * max_nodes:
            break
        _, logits = drafter.verify_tree(dkv, tokens, parents, base_pos, want_logits=True)
        rows = logits[torch.tensor(frontier, device=logits.device)].contiguous()
        idx, val, lse = drafter.topk(rows, width)
        lp = (val - lse[:, None]).tolist()
        nxt = []
        for r, f in enumerate(frontier):
            for t, v in zip(idx[r].tolist(), lp[r]):
                tokens.append(int(t))
                parents.append(f)
                cum.append(cum[f] + float(v))
                nxt.append(len(tokens) - 1)
        frontier = nxt
    keep = sorted(sorted(range(len(tokens)), key=lambda i: (-cum[i], i))[:max_nodes])
    pos = {old: new for new, old in enumerate(keep)}
    k_tokens = [tokens[i] for i in keep]
    k_parents = [pos[parents[i]] if parents[i] >= 0 else -1 for i in keep]
    children = [0] * len(keep)
    for p in k_parents:
        if p >= 0:
            children[p] += 1
    paths = []
    for i in range(len(keep)):
        if children[i] == 0:                 # a leaf: its root-to-leaf path
            path, j = [], i
            while j >= 0:
                path.append(k_tokens[j])
                j = k_parents[j]
            paths.append(path[::-1])
    return SpeculativeForest.build(paths)


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    verify_ms: List[float] = field(default_factory=list)


def speculative_generate(target, drafter, prompt: Sequence[int], n_new: int, branching=(4, 2, 1, 1),
                         max_nodes: int = 16, capacity: Optional[int] = None):
    """Greedy speculative decoding: the drafter proposes a tree, the target verifies all of it in one
    batched pass (`verify_tree`), the reference's selection rule picks the emitted tokens, the
    accepted nodes' K/V are committed. Lossless: the tokens equal plain greedy decoding of the
    target. Returns (tokens, SpecStats); `verify_ms` holds the device time of every verify pass."""
    import torch
    cap = capacity or len(prompt) + n_new + 8 * max_nodes
    tkv, dkv = target.new_kv(cap), drafter.new_kv(cap)
    _, am = target.forward(tkv, list(prompt), want_logits=False, last_only=True)
    root_pred = int(am[-1])
    d_logits, _ = drafter.forward(dkv, list(prompt), last_only=True)
    d_root = d_logits[-1]
    out: List[int] = []
    stats = SpecStats()
    stream = torch.cuda.current_stream(target.device)
    while len(out) < n_new:
        base = tkv.length
        forest = draft_tree(drafter, dkv, d_root, base, branching, max_nodes)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        res = verify_tree(target, tkv, forest, root_pred, base)
        e1.record(stream)
        ver = res.verification
        commit_tree(target, tkv, res)
        stats.rounds += 1
        stats.drafted += forest.node_count
        stats.accepted += ver.accepted_draft_tokens
        e1.synchronize()
        stats.verify_ms.append(e0.elapsed_time(e1))
        emitted = list(ver.emitted)
        if ver.rejected:                     # the target's own token at the mismatch: feed it
            _, am = target.forward(tkv, [emitted[-1]], want_logits=False)
            root_pred = int(am[-1])
        elif res.next_pred is not None:
            root_pred = res.next_pred
        else:                                # empty forest: the emitted token is the root prediction
            _, am = target.forward(tkv, [emitted[-1]], want_logits=False)
            root_pred = int(am[-1])
        dkv.length = base
        d_logits, _ = drafter.forward(dkv, emitted, last_only=True)
        d_root = d_logits[-1]
        out.extend(emitted)
    tkv.close()
    dkv.close()
    return out[:n_new], stats
