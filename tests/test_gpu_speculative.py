"""The speculative decode loop on the GPU (cfg2 mechanics on small shapes): the device top-k
against torch.topk / logsumexp (ties -> lower index), the drafter tree's shape, and greedy
speculative decoding producing exactly the target's greedy tokens (it is lossless)."""
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights, random_prompt, truncate

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair():
    from dataclasses import replace
    from seedplane_b200.engine import CudaQwen2
    cfg = replace(PRESETS["tiny-hd128"], layers=4, name="tiny-4l")
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    dcfg = replace(cfg, layers=1, name="tiny-draft")
    target = CudaQwen2(cfg, w, device="cuda:0")
    drafter = CudaQwen2(dcfg, truncate(w, cfg, 1), device="cuda:0")
    yield cfg, w, target, drafter
    target.close()
    drafter.close()


def test_topk_matches_torch(pair):
    cfg, w, target, drafter = pair
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(5, 3001, device="cuda", generator=g)
    x[2, 100] = x[2, 7] = 50.0                  # a tie: the lower index comes first
    x[3, :] = -float("inf")
    x[3, 9] = 1.0
    for k in (1, 2, 3, 4, 6, 8):
        idx, val, lse = target.topk(x, k)
        for r in range(5):
            row = x[r].cpu().double()
            order = sorted(range(row.numel()), key=lambda i: (-float(row[i]), i))[:k]
            assert idx[r].tolist() == order if r != 3 else idx[r, 0].item() == 9
            assert torch.allclose(val[r].cpu().double(), row[order], atol=0) or r == 3
            assert abs(float(lse[r]) - float(torch.logsumexp(row, 0))) < 1e-4


def test_draft_tree_shape(pair):
    from seedplane_b200.speculative import draft_tree
    cfg, w, target, drafter = pair
    prompt = random_prompt(cfg.vocab, 20, seed=3)
    dkv = drafter.new_kv(256)
    logits, _ = drafter.forward(dkv, prompt)
    forest = draft_tree(drafter, dkv, logits[-1], len(prompt), (4, 2, 1, 1), 16)
    flat = forest.flatten()
    assert 1 <= len(flat.tokens) <= 16 and max(flat.depths) <= 4
    assert all(p < i for i, p in enumerate(flat.parents))
    assert dkv.length == len(prompt)            # tree nodes do not advance the drafter cache
    dkv.close()


def test_speculative_greedy_is_lossless(pair):
    from seedplane_b200.speculative import speculative_generate
    cfg, w, target, drafter = pair
    # seed 6: the oracle's top-1 / top-2 margin stays above 0.03 for 40 steps, so no numerical tie can
    # flip a token (the verify pass and the oracle sum in different orders)
    prompt = random_prompt(cfg.vocab, 17, seed=6)
    want, margins = OracleQwen2(cfg, w, kv_fp16=True).greedy(prompt, 30)
    assert min(margins) > 0.02
    got, stats = speculative_generate(target, drafter, prompt, 30)
    assert got == want
    assert stats.rounds >= 1 and len(stats.verify_ms) == stats.rounds
    target.status()
    drafter.status()


@pytest.mark.parametrize("V", [5000, 151936])
def test_stochastic_accept_matches_oracle(pair, V):
    """The device's stochastic acceptance takes the oracle's decisions bit for bit (same fp64
    arithmetic, summation order and RNG), on random trees and logits."""
    import numpy as np
    from oracle.speculative_oracle import accept_stochastic as ref
    from seedplane_b200.speculative import SpeculativeForest, accept_stochastic
    cfg, w, target, drafter = pair
    rng = np.random.default_rng(V)
    cases = 0
    for trial in range(4):
        paths = [[int(rng.integers(0, V)) for _ in range(int(rng.integers(1, 5)))] for _ in range(5)]
        flat = SpeculativeForest.build(paths).flatten()
        n = len(flat.tokens)
        t = (rng.normal(size=(n + 1, V)) * 3).astype(np.float32)
        d = (rng.normal(size=(n + 1, V)) * 3).astype(np.float32)
        # make the drafts likely under both, so acceptances happen
        for i, tok in enumerate(flat.tokens):
            row = flat.parents[i] + 1
            t[row, tok] += 6.0
            d[row, tok] += 6.5
        td, dd = torch.from_numpy(t).cuda(), torch.from_numpy(d).cuda()
        for seed, counter in ((1, 0), (1, 1), (99, 7), (2 ** 40 + 3, 123)):
            ver, nodes = accept_stochastic(target, flat, td, dd, 1.0 if trial % 2 == 0 else 0.7, seed, counter)
            want_tokens, want_nodes = ref(list(flat.tokens), list(flat.parents), t, d,
                                          1.0 if trial % 2 == 0 else 0.7, seed, counter)
            assert list(ver.emitted) == want_tokens and list(nodes) == want_nodes
            cases += 1
    assert cases == 16


def test_accept_greedy_device_matches_host_rule(pair):
    """sp_accept_greedy (the decision on the device from device-resident argmaxes) equals the host
    selection and the oracle's restatement of verify_greedy (speculative.py:55-92) on random
    forests: shared prefixes, duplicate branches, branches that are prefixes of others, ties."""
    import random
    from oracle import speculative_oracle as so
    from seedplane_b200.speculative import SpeculativeForest, accept_greedy, accept_greedy_device
    cfg, w, target, drafter = pair
    rng = random.Random(7)
    for case in range(300):
        vocab = rng.choice((3, 5, 50))
        branches = []
        for _ in range(rng.randint(0, 8)):
            b = [rng.randrange(vocab) for _ in range(rng.randint(0, 5))]
            if branches and rng.random() < 0.3:
                b = list(rng.choice(branches))[:rng.randint(0, 5)]      # a duplicate or a prefix
            branches.append(b)
        forest = SpeculativeForest.build(branches)
        flat = forest.flatten()
        if len(flat.tokens) > 64:
            continue
        root = rng.randrange(vocab)
        # predictions that often agree with a child so that paths get accepted
        pred = []
        for i in range(len(flat.tokens)):
            kids = [j for j, p in enumerate(flat.parents) if p == i]
            pred.append(flat.tokens[rng.choice(kids)] if kids and rng.random() < 0.7 else rng.randrange(vocab))
        if flat.tokens and rng.random() < 0.7:
            root = rng.choice([flat.tokens[j] for j, p in enumerate(flat.parents) if p < 0])
        dev = torch.tensor(pred if pred else [0], dtype=torch.int32, device="cuda:0")
        ver_d, nodes_d, nxt = accept_greedy_device(target, flat, root, dev)
        ver_h, nodes_h = accept_greedy(flat, root, pred)
        assert (ver_d, nodes_d) == (ver_h, nodes_h), case
        want_next = pred[nodes_h[-1]] if nodes_h and not ver_h.rejected else None
        assert nxt == want_next, case
        want = so.accept_from_predictions(list(flat.paths), [list(p) for p in flat.node_paths], list(flat.tokens),
                                          root, pred)
        assert (tuple(ver_h.emitted), ver_h.accepted_draft_tokens, ver_h.rejected, ver_h.target_steps,
                tuple(ver_h.branch)) == tuple(want), case
