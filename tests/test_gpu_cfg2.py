"""Parity on the cfg2 shapes: the Qwen2-0.5B-shaped fp16 target after a 128-token prompt, draft trees
of 16 nodes (branching 4, 2, 1, 1, depth 4), the 2-layer drafter, 64 output tokens.

* one batched verify pass against the oracle's masked pass over the same tree (every node sees the
  prompt and its own ancestors, position = prompt length + depth - 1): logits within 1e-2 relative
  of the row's scale, argmaxes equal where the oracle's top-1 / top-2 margin is not a numerical
  tie, and the accepted path equal to the reference rule (`verify_greedy`, speculative.py:55-92)
  applied to the oracle's own node predictions, decided on the device and on the host;
* greedy speculative decoding for 64 tokens equal to the target's plain greedy tokens and the
  oracle's (the loop is lossless).
"""
import random

import pytest
import torch

from oracle import speculative_oracle as so
from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import QWEN2_0_5B
from seedplane_b200.randinit import make_weights, random_prompt, truncate

pytestmark = pytest.mark.gpu
PROMPT, NODES = 128, 16


@pytest.fixture(scope="module")
def cfg2():
    from dataclasses import replace
    from seedplane_b200.engine import CudaQwen2
    cfg = QWEN2_0_5B
    w = make_weights(cfg, seed=0, dtype=torch.float16)
    target = CudaQwen2(cfg, w, device="cuda:0")
    dcfg = replace(cfg, layers=2, name="qwen2-0.5b-draft2")
    drafter = CudaQwen2(dcfg, truncate(w, cfg, 2), device="cuda:0")
    oracle = OracleQwen2(cfg, w, kv_fp16=True)
    prompt = random_prompt(cfg.vocab, PROMPT, seed=0)
    greedy, margins = oracle.greedy(prompt, 64, capacity=PROMPT + 80)
    yield cfg, w, target, drafter, oracle, prompt, greedy, margins
    target.close()
    drafter.close()


def _tree_4211(rng, vocab, chain=None):
    """16 nodes of branching 4, 2, 1, 1 at depth 4: the 4 roots, 2 children for each of the first
    3 roots, then one child for each of the first 3 nodes of each deeper level (4 + 6 + 3 + 3),
    an ancestor-closed cut like the drafter's best-first one. With `chain`, the first child along
    the first branch carries those tokens (so a path can be accepted)."""
    tokens, parents, depth, level, on = [], [], [], [-1], {-1}
    for d, (width, expand) in enumerate(((4, 1), (2, 3), (1, 3), (1, 3))):
        nxt = []
        for par in level[:expand]:
            for c in range(width):
                carry = chain is not None and c == 0 and par in on and d < len(chain)
                tokens.append(chain[d] if carry else rng.randrange(vocab))
                parents.append(par)
                depth.append(d + 1)
                if carry:
                    on.add(len(tokens) - 1)
                nxt.append(len(tokens) - 1)
        level = nxt
    assert len(tokens) == NODES and max(depth) == 4
    return tokens, parents, depth


def _oracle_tree(oracle, prompt, tokens, parents, depth):
    cache = oracle.new_cache(PROMPT + NODES + 8)
    oracle.forward(prompt, cache)
    n = len(tokens)
    vis = torch.zeros(n, PROMPT + n, dtype=torch.bool)
    vis[:, :PROMPT] = True
    for i in range(n):
        j = i
        while j >= 0:
            vis[i, PROMPT + j] = True
            j = parents[j]
    logits, _ = oracle.forward(tokens, cache, all_logits=True, positions=[PROMPT + d - 1 for d in depth],
                               visible=vis, advance=False)
    return logits


@pytest.mark.parametrize("with_chain", [False, True])
def test_cfg2_tree_verify_16_nodes(cfg2, with_chain):
    from seedplane_b200.speculative import SpeculativeForest, accept_greedy, accept_greedy_device
    cfg, w, target, drafter, oracle, prompt, greedy, margins = cfg2
    rng = random.Random(11 + with_chain)
    tokens, parents, depth = _tree_4211(rng, cfg.vocab, greedy[:4] if with_chain else None)
    kv = target.new_kv(PROMPT + NODES + 8)
    _, am = target.forward(kv, prompt, want_logits=False)
    root = int(am[-1])
    assert root == greedy[0]
    argmax, logits = target.verify_tree(kv, tokens, parents, base_pos=PROMPT, want_logits=True)
    assert kv.length == PROMPT
    want = _oracle_tree(oracle, prompt, tokens, parents, depth)
    got = logits.float().cpu()
    for i in range(len(tokens)):
        scale = float(want[i].abs().max())
        err = float((got[i] - want[i]).abs().max())
        assert err <= 1e-2 * scale, (i, err, scale)
        top = torch.topk(want[i], 2).values
        if float(top[0] - top[1]) > 1e-3 * scale:
            assert int(argmax[i]) == int(want[i].argmax()), i
    # the accepted path: the oracle's node predictions through the reference's rule
    paths, j_leaf = [], set(range(len(tokens))) - set(parents)
    for leaf in sorted(j_leaf):
        p, j = [], leaf
        while j >= 0:
            p.append(tokens[j])
            j = parents[j]
        paths.append(p[::-1])
    forest = SpeculativeForest.build(paths)
    flat = forest.flatten()
    remap = {}
    for fi in range(len(flat.tokens)):            # flat node -> the tree node with the same path
        p, j = [], fi
        while j >= 0:
            p.append(flat.tokens[j])
            j = flat.parents[j]
        remap[fi] = next(i for i in range(len(tokens)) if _path(tokens, parents, i) == p[::-1])
    pred_oracle = [int(want[remap[fi]].argmax()) for fi in range(len(flat.tokens))]
    ref = so.accept_from_predictions(list(flat.paths), [list(p) for p in flat.node_paths], list(flat.tokens),
                                     greedy[0], pred_oracle)
    pred_dev = argmax[torch.tensor([remap[fi] for fi in range(len(flat.tokens))], device=argmax.device)]
    ver_d, nodes_d, _ = accept_greedy_device(target, flat, root, pred_dev.contiguous())
    ver_h, _ = accept_greedy(flat, root, pred_dev.cpu().tolist())
    assert ver_d == ver_h
    assert (tuple(ver_d.emitted), ver_d.accepted_draft_tokens, ver_d.rejected, ver_d.target_steps,
            tuple(ver_d.branch)) == tuple(ref)
    if with_chain:
        assert ver_d.accepted_draft_tokens == 4 and list(ver_d.emitted) == greedy[:4]
    kv.close()
    target.status()


def _path(tokens, parents, i):
    p = []
    while i >= 0:
        p.append(tokens[i])
        i = parents[i]
    return p[::-1]


def test_cfg2_speculative_64_tokens(cfg2):
    from seedplane_b200.speculative import speculative_generate
    cfg, w, target, drafter, oracle, prompt, greedy, margins = cfg2
    kv = target.new_kv(PROMPT + 80)
    _, am = target.forward(kv, prompt, want_logits=False)
    first = int(am[-1])
    rest, _ = target.decode(kv, first, PROMPT, 63)
    plain = [first] + rest.cpu().tolist()
    kv.close()
    got, stats = speculative_generate(target, drafter, prompt, 64, branching=(4, 2, 1, 1), max_nodes=NODES)
    assert got == plain
    d = next((i for i, (a, b) in enumerate(zip(plain, greedy)) if a != b), None)
    assert d is None, (d, margins[d] if d is not None else None)
    assert stats.rounds >= 1
    target.status()
    drafter.status()
