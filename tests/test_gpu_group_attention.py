"""GQA attention on the tensor cores, in both passes.

The step kernel's grouped attention items: one item per (kv head, context chunk) computing all q
heads of the GQA group on the tensor cores (scores and values as m16n8 MMAs with fp16 hi / lo
rows), selected from `SEEDPLANE_ATTN_GROUP_CTX` visible positions on. The batched pass's attention
(prompt chunks and verify trees) by GQA group and key chunk, with the chunks' partials merged.

Every case runs the prompt through the step kernel too (`SEEDPLANE_PREFILL=steps`), so each prompt
token is one step with its own context length: chunks of one tile, partial tiles, the step's own
K/V row at every position of a tile. Capping the chunks (`SEEDPLANE_ATTN_GROUP_CHUNKS=2`) gives
each warp many tiles. Tree verification through steps checks the ancestor masks. Bars: greedy
tokens identical to the oracle's; logits within 1e-3 of the largest |logit|.
"""
import numpy as np
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights, random_prompt

pytestmark = pytest.mark.gpu


def _close(got, want, rel=1e-3):
    got = got.detach().float().cpu().numpy()
    want = want.detach().float().cpu().numpy()
    err = float(np.abs(got - want).max())
    assert err <= rel * float(np.abs(want).max()), f"max |err| {err:.3e}"


@pytest.mark.parametrize("chunks", ["64", "2"])
@pytest.mark.parametrize("name", ["tiny-hd64", "tiny-hd128"])
def test_grouped_items_decode_matches_oracle(monkeypatch, name, chunks):
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[name]
    monkeypatch.setenv("SEEDPLANE_ATTN_GROUP_CTX", "0")
    monkeypatch.setenv("SEEDPLANE_ATTN_GROUP_CHUNKS", chunks)
    monkeypatch.setenv("SEEDPLANE_PREFILL", "steps")
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    prompt = random_prompt(cfg.vocab, 150, seed=4)
    eng = CudaQwen2(cfg, w, device="cuda:0")
    kv = eng.new_kv(256)
    logits, argmax = eng.forward(kv, prompt, all_logits=True)
    first = int(argmax[-1])
    out, last = eng.decode(kv, first, len(prompt), 19, want_logits=True)
    got = [first] + out.cpu().tolist()
    eng.status()
    eng.close()
    o = OracleQwen2(cfg, w, kv_fp16=True)
    want_all, _ = o.forward(prompt, o.new_cache(256), all_logits=True)
    _close(logits, want_all)
    want, margins = o.greedy(prompt, 20, capacity=256)
    assert got == want, f"min margin {min(margins):.4f}"
    _close(last, o.prefix_logits(prompt + want[:-1]))


@pytest.mark.parametrize("name", ["tiny-hd64", "tiny-hd128"])
def test_grouped_items_tree_verify_through_steps(monkeypatch, name):
    """A 12-node tree verified one node per step: node i sees the prompt and its ancestors only."""
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[name]
    monkeypatch.setenv("SEEDPLANE_ATTN_GROUP_CTX", "0")
    monkeypatch.setenv("SEEDPLANE_PREFILL", "steps")
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    o = OracleQwen2(cfg, w, kv_fp16=True)
    eng = CudaQwen2(cfg, w, device="cuda:0")
    try:
        rng = np.random.default_rng(3)
        prompt = random_prompt(cfg.vocab, 37, seed=6)
        parents = [-1] + [int(rng.integers(-1, i)) for i in range(1, 12)]
        tokens = [int(t) for t in rng.integers(0, cfg.vocab, size=12)]
        kv = eng.new_kv(64)
        eng.forward(kv, prompt, want_logits=False)
        argmax, logits = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt), want_logits=True)
        for i in range(12):
            path, j = [], i
            while j >= 0:
                path.append(tokens[j])
                j = parents[j]
            want = o.prefix_logits(prompt + path[::-1])
            _close(logits[i], want)
            assert int(argmax[i]) == int(want.argmax())
        eng.status()
    finally:
        eng.close()


def test_grouped_and_per_head_items_agree_on_qwen2_0_5b(monkeypatch):
    """The 0.5B shape (14 q / 2 kv heads of 64 dims: groups of 7): 48 greedy tokens after a
    700-token prompt with grouped items from the first step on, against the per-head items: the
    same tokens (fp32-grade sums in both) and last logits within 1e-3."""
    from seedplane_b200.config import QWEN2_0_5B
    from seedplane_b200.engine import CudaQwen2
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    prompt = random_prompt(QWEN2_0_5B.vocab, 700, seed=2)
    runs = {}
    for ctx in ("0", str(1 << 30)):
        monkeypatch.setenv("SEEDPLANE_ATTN_GROUP_CTX", ctx)
        eng = CudaQwen2(QWEN2_0_5B, w, device="cuda:0")
        try:
            kv = eng.new_kv(800)
            _, am = eng.forward(kv, prompt, want_logits=False)
            first = int(am[-1])
            out, last = eng.decode(kv, first, len(prompt), 47, want_logits=True)
            runs[ctx] = ([first] + out.cpu().tolist(), last.float().cpu())
            eng.status()
        finally:
            eng.close()
    (g_tok, g_last), (h_tok, h_last) = runs["0"], runs[str(1 << 30)]
    assert g_tok == h_tok
    _close(g_last, h_last)


@pytest.mark.parametrize("name", ["tiny-hd64", "tiny-hd128"])
def test_batched_pass_attention_over_several_key_chunks(name):
    """A 400-token prompt in one batched pass (causal; 400 keys cut into two chunks of 256 and the
    partials merged) and a 12-node tree verified after it (keys of the prefix in two chunks, the
    nodes' ancestor masks; a cache of 1,100 slots, so the tree takes the grouped kernel too):
    every prompt row's logits and every node's logits and argmax against the oracle."""
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[name]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    o = OracleQwen2(cfg, w, kv_fp16=True)
    eng = CudaQwen2(cfg, w, device="cuda:0")
    try:
        prompt = random_prompt(cfg.vocab, 400, seed=9)
        kv = eng.new_kv(1100)
        logits, _ = eng.forward(kv, prompt, all_logits=True)
        want_all, _ = o.forward(prompt, o.new_cache(512), all_logits=True)
        _close(logits, want_all)
        rng = np.random.default_rng(5)
        parents = [-1] + [int(rng.integers(-1, i)) for i in range(1, 12)]
        tokens = [int(t) for t in rng.integers(0, cfg.vocab, size=12)]
        argmax, tl = eng.verify_tree(kv, tokens, parents, base_pos=len(prompt), want_logits=True)
        for i in range(12):
            path, j = [], i
            while j >= 0:
                path.append(tokens[j])
                j = parents[j]
            want = o.prefix_logits(prompt + path[::-1])
            _close(tl[i], want)
            assert int(argmax[i]) == int(want.argmax())
        eng.status()
    finally:
        eng.close()
