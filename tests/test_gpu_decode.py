"""Parity of the CUDA decode path (through the C ABI) with the CPU oracle.

The oracle runs the same fp16-rounded checkpoint in fp32 with K/V rounded to fp16 at cache write,
which is what the engine stores. Bars: greedy tokens identical; logits within 1e-3 of the largest
|logit| (the product bar is 1e-2 relative, fp16 weights with fp32 accumulation)."""
import numpy as np
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from oracle import speculative_oracle as so
from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights, random_prompt

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


def assert_logits_close(got, want, rel=LOGIT_TOL):
    got = got.detach().float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    want = want.detach().float().cpu().numpy() if isinstance(want, torch.Tensor) else np.asarray(want)
    err = float(np.abs(got - want).max())
    scale = float(np.abs(want).max())
    assert err <= rel * scale, f"max |err| {err:.3e} > {rel} x max|logit| {scale:.3e}"


@pytest.fixture(scope="module", params=["tiny-hd64", "tiny-hd128", "tiny-untied"])
def tiny(request):
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[request.param]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    eng = CudaQwen2(cfg, w, device="cuda:0")
    yield cfg, w, eng, OracleQwen2(cfg, w, kv_fp16=True)
    eng.close()


def test_prefill_all_logits(tiny):
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    kv = eng.new_kv(64)
    logits, argmax = eng.forward(kv, prompt, all_logits=True)
    want, _ = o.forward(prompt, o.new_cache(64), all_logits=True)
    assert_logits_close(logits, want)
    assert argmax.cpu().tolist() == want.argmax(-1).tolist()
    assert kv.length == len(prompt)
    eng.status()


def test_last_row_logits_and_positions(tiny):
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 9, seed=3)
    pos = [p + 40 for p in range(len(prompt))]
    kv = eng.new_kv(32)
    logits, _ = eng.forward(kv, prompt, positions=pos)
    want, _ = o.forward(prompt, o.new_cache(32), positions=pos)
    assert logits.shape == (1, cfg.vocab)
    assert_logits_close(logits, want)
    eng.status()


def test_greedy_decode_matches_oracle(tiny):
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    want, margins = o.greedy(prompt, 24, capacity=64)
    kv = eng.new_kv(64)
    _, argmax = eng.forward(kv, prompt, want_logits=False)
    first = int(argmax[-1])
    out, logits = eng.decode(kv, first, len(prompt), 23, want_logits=True)
    got = [first] + out.cpu().tolist()
    assert got == want, f"min margin {min(margins):.4f}"
    assert kv.length == len(prompt) + 23
    eng.status()


def test_chunked_prefill_and_decode_logits(tiny):
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    kv = eng.new_kv(64)
    eng.forward(kv, prompt[:7], want_logits=False)
    logits, _ = eng.forward(kv, prompt[7:], all_logits=True)
    c = o.new_cache(64)
    o.forward(prompt[:7], c)
    want, c = o.forward(prompt[7:], c, all_logits=True)
    assert_logits_close(logits, want)
    # one decode step with logits
    nxt = int(want[-1].argmax())
    out, lg = eng.decode(kv, nxt, kv.length, 1, want_logits=True)
    want2, _ = o.forward([nxt], c)
    assert_logits_close(lg, want2[0])
    assert int(out[0]) == int(want2[0].argmax())
    eng.status()


def _random_tree(rng, n, vocab):
    parents, tokens = [], []
    for i in range(n):
        parents.append(-1 if i == 0 or rng.random() < 0.2 else int(rng.integers(0, i)))
        tokens.append(int(rng.integers(0, vocab)))
    return tokens, parents


def test_tree_verify_matches_prefix_forwards(tiny):
    cfg, w, eng, o = tiny
    rng = np.random.default_rng(1)
    prompt = random_prompt(cfg.vocab, 10, seed=5)
    tokens, parents = _random_tree(rng, 12, cfg.vocab)
    kv = eng.new_kv(64)
    eng.forward(kv, prompt, want_logits=False)
    argmax, logits = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt), want_logits=True)
    assert kv.length == len(prompt)
    for i in range(len(tokens)):
        path, j = [], i
        while j >= 0:
            path.append(tokens[j])
            j = parents[j]
        want = o.prefix_logits(prompt + path[::-1])
        assert_logits_close(logits[i], want)
        assert int(argmax[i]) == int(want.argmax())
    eng.status()


def test_commit_accepted_path_then_continue(tiny):
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 10, seed=6)
    greedy, _ = o.greedy(prompt, 5, capacity=64)
    # tree: a wrong sibling first, then the greedy chain (nodes 1, 2, 4 form the accepted path)
    tokens = [(greedy[0] + 1) % cfg.vocab, greedy[0], greedy[1], (greedy[2] + 3) % cfg.vocab, greedy[2]]
    parents = [-1, -1, 1, 2, 2]
    kv = eng.new_kv(64)
    eng.forward(kv, prompt, want_logits=False)
    argmax, _ = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt))
    assert [int(argmax[i]) for i in (1, 2, 4)] == greedy[1:4]
    base = kv.length
    eng.kv_commit(kv, [base + 1, base + 2, base + 4])
    assert kv.length == base + 3
    out, _ = eng.decode(kv, greedy[3], kv.length, 1)
    assert int(out[0]) == greedy[4]
    eng.status()


def test_errors_are_reported_not_faulted(tiny):
    cfg, w, eng, o = tiny
    kv = eng.new_kv(8)
    with pytest.raises(ValueError):
        eng.forward(kv, list(range(9)))
    with pytest.raises(ValueError):
        eng.forward(kv, [])
    with pytest.raises(ValueError):
        eng.decode(kv, cfg.vocab + 5, 0, 1)
    # an out-of-vocabulary id inside a device array is clamped and recorded by the kernel
    eng.forward(kv, [cfg.vocab + 7], want_logits=False)
    from seedplane_b200._native import EngineError
    with pytest.raises(EngineError, match="vocabulary"):
        eng.status()
    eng.status()  # cleared


def test_qwen2engine_surface_generate(tiny):
    from seedplane_b200.qwen_engine import Qwen2Engine
    cfg, w, eng, o = tiny
    e = Qwen2Engine(config=cfg, weights=w)
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    want, _ = o.greedy(prompt, 20, capacity=64)
    assert list(e.generate(prompt, max_new_tokens=20, block=7)) == want
    logits, cache = e.forward(prompt, e.new_cache(64), all_logits=True)
    assert cache.length == len(prompt) and logits.shape == (len(prompt), cfg.vocab)
    cache.length = 5                      # rollback, then re-feed: same logits
    l2, _ = e.forward(prompt[5:], cache, all_logits=True)
    assert_logits_close(l2, logits[5:])
    with pytest.raises(ValueError):
        e.forward([], cache)
    with pytest.raises(ValueError):
        e.forward([1, 2], cache, positions=[1])
    e.engine.close()


def argmax_cases(seed=0):
    """Logit matrices with planted ties and maxima at chunk edges; numpy's argmax (first index of
    the maximum) is the oracle, as torch.argmax / `sample` in the reference."""
    g = np.random.default_rng(seed)
    cases = []
    for rows, cols, ld in ((1, 151936, 151936), (3, 1000, 1000), (70, 1200, 1204), (5, 8193, 8195), (2, 7, 7)):
        x = g.standard_normal((rows, ld)).astype(np.float32)
        for r in range(rows):
            j = int(g.integers(0, cols))
            x[r, j] = 9.0
            k = int(g.integers(0, cols))
            x[r, k] = 9.0                       # a tie: the lower index must win
            if r % 3 == 0:
                x[r, cols - 1] = 9.5            # maximum in the last column of the row
            x[r, cols:] = 100.0                 # padding beyond `cols` must be ignored
        cases.append((x, cols))
    return cases


def test_argmax_rows_first_index(tiny):
    cfg, w, eng, o = tiny
    for x, cols in argmax_cases():
        dev = torch.from_numpy(x).to(eng.device)
        got = eng.argmax(dev[:, :cols]).cpu().numpy()
        want = np.argmax(x[:, :cols], axis=1)
        assert (got == want).all()


def test_speculative_surface_verify_tree_and_commit(tiny):
    """`speculative.verify_tree` (one batched device pass) takes the same decision as the
    reference's sequential `verify_greedy` with the oracle as target; after `commit_tree` the
    cache continues exactly like the oracle on the committed tokens."""
    from seedplane_b200.speculative import SpeculativeForest, commit_tree, verify_greedy, verify_tree
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, 10, seed=3)
    greedy, _ = o.greedy(prompt, 6, capacity=64)
    V = cfg.vocab

    def target(prefix):
        lg, _ = o.forward(list(prefix), o.new_cache(64))
        return lg[-1].tolist()

    for branches in ([greedy[:4], greedy[:2] + [(greedy[2] + 1) % V], [(greedy[0] + 3) % V], greedy[:3]],
                     [[(greedy[0] + 1) % V, greedy[1]], greedy[:1] + [(greedy[1] + 7) % V]],
                     [greedy[:5]]):
        kv = eng.new_kv(64)
        _, am = eng.forward(kv, prompt, want_logits=False)
        root = int(am[-1])
        assert root == greedy[0]
        forest = SpeculativeForest.build(branches)
        res = verify_tree(eng, kv, forest, root_pred=root, base_pos=len(prompt))
        assert res.verification == verify_greedy(prompt, forest, target)
        n_acc = res.verification.accepted_draft_tokens
        assert commit_tree(eng, kv, res) == len(prompt) + n_acc
        # continue from the committed prefix: feed the last emitted token (correction or last
        # accepted) unless it is already in the cache
        emitted = list(res.verification.emitted)
        if res.verification.rejected:
            toks, _ = eng.decode(kv, emitted[-1], len(prompt) + n_acc, 2)
            want, _ = o.greedy(prompt + emitted, 2, capacity=64)
        else:
            assert res.next_pred == greedy[len(emitted)]
            toks, _ = eng.decode(kv, res.next_pred, len(prompt) + n_acc, 2)
            want, _ = o.greedy(prompt + emitted + [res.next_pred], 2, capacity=64)
        assert toks.cpu().tolist() == want
        kv.close()


@pytest.mark.parametrize("n", [1, 5, 12, 70])
def test_last_only_forward_gives_the_last_tokens_head(tiny, n):
    """sp_forward with all_logits = 2 (the last token's LM head alone) gives the same logits and
    argmax as the full forward's last row, through the step path (n < 8) and the batched pass."""
    cfg, w, eng, o = tiny
    prompt = random_prompt(cfg.vocab, n, seed=3)
    kv1, kv2 = eng.new_kv(96), eng.new_kv(96)
    try:
        lg_all, am_all = eng.forward(kv1, prompt, all_logits=True)
        lg, am = eng.forward(kv2, prompt, last_only=True)
        assert am.numel() == 1 and int(am[0]) == int(am_all[-1])
        assert_logits_close(lg[0], lg_all[-1], rel=1e-6)
        assert kv2.length == n
        want, _ = o.forward(prompt, o.new_cache(96))
        assert_logits_close(lg[0], want[-1])
    finally:
        kv1.close()
        kv2.close()
