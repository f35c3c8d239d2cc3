"""Blockwise-int8 weights through the step kernel's dequantizing GEMV, against the oracle.

The checkpoint format is int8 values with one fp16 scale per 32 inputs of a row (w = q * scale,
exact in fp32). The oracle runs the same checkpoint dequantized to fp32, with K/V rounded to fp16
at cache write as the engine stores them. Bars: greedy tokens identical; logits within 1e-3 of
the largest |logit| (fp16 hi/lo activations and fp32 block sums against an fp32 matvec).

The tied tiny models mix formats (int8 layers, fp16 embedding as the LM head); the untied one
streams an int8 LM head too. Prompts of 8 or more tokens and tree verifies go through the batched
pass, whose GEMMs use exact fp16 hi / lo halves of the dequantized weights; shorter prompts, decode
and `SEEDPLANE_PREFILL=steps` go through the step kernel's int8 units.
"""
import numpy as np
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS, QWEN2_0_5B
from seedplane_b200.randinit import make_int8_blockwise, random_prompt

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


def assert_logits_close(got, want, rel=LOGIT_TOL):
    got = got.detach().float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    want = want.detach().float().cpu().numpy() if isinstance(want, torch.Tensor) else np.asarray(want)
    err = float(np.abs(got - want).max())
    scale = float(np.abs(want).max())
    assert err <= rel * scale, f"max |err| {err:.3e} > {rel} x max|logit| {scale:.3e}"


@pytest.fixture(scope="module", params=["tiny-hd64", "tiny-hd128", "tiny-untied"])
def tiny8(request):
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[request.param]
    w = make_int8_blockwise(cfg, seed=0, std=0.1)
    eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
    yield cfg, w, eng, OracleQwen2(cfg, w, kv_fp16=True)
    eng.close()


def test_int8_prompt_all_logits(tiny8):
    cfg, w, eng, o = tiny8
    prompt = random_prompt(cfg.vocab, 12, seed=0)
    kv = eng.new_kv(64)
    logits, argmax = eng.forward(kv, prompt, all_logits=True)
    want, _ = o.forward(prompt, o.new_cache(64), all_logits=True)
    assert_logits_close(logits, want)
    assert argmax.cpu().tolist() == want.argmax(-1).tolist()
    eng.status()


def test_int8_greedy_decode_matches_oracle(tiny8):
    cfg, w, eng, o = tiny8
    prompt = random_prompt(cfg.vocab, 12, seed=1)
    want, margins = o.greedy(prompt, 24, capacity=64)
    kv = eng.new_kv(64)
    _, argmax = eng.forward(kv, prompt, want_logits=False)
    first = int(argmax[-1])
    out, logits = eng.decode(kv, first, len(prompt), 23, want_logits=True)
    got = [first] + out.cpu().tolist()
    assert got == want, f"min margin {min(margins):.4f}"
    # the last step's logits too
    want_last = o.prefix_logits(prompt + want[:-1])
    assert_logits_close(logits, want_last)
    eng.status()


def test_int8_tree_verify_matches_prefix_forwards(tiny8):
    cfg, w, eng, o = tiny8
    rng = np.random.default_rng(2)
    prompt = random_prompt(cfg.vocab, 9, seed=5)
    tokens, parents = [], []
    for i in range(10):
        parents.append(-1 if i == 0 or rng.random() < 0.2 else int(rng.integers(0, i)))
        tokens.append(int(rng.integers(0, cfg.vocab)))
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


def test_int8_qwen2_0_5b_shape_greedy():
    """The 0.5B architecture with the benchmark's int8 recipe (scale ~ |N(0, 0.02)| / 127)."""
    from seedplane_b200.engine import CudaQwen2
    cfg = QWEN2_0_5B
    w = make_int8_blockwise(cfg, seed=0)
    prompt = random_prompt(cfg.vocab, 16, seed=0)
    eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
    kv = eng.new_kv(64)
    logits, argmax = eng.forward(kv, prompt)
    first = int(argmax[-1])
    out, _ = eng.decode(kv, first, len(prompt), 11)
    got = [first] + out.cpu().tolist()
    eng.close()
    o = OracleQwen2(cfg, w, kv_fp16=True)
    want, margins = o.greedy(prompt, 12, capacity=64)
    want_logits = o.prefix_logits(prompt)
    assert_logits_close(logits[0], want_logits)
    d = next((i for i, (x, y) in enumerate(zip(got, want)) if x != y), None)
    assert d is None, f"first divergence at {d}: margin there {margins[d]:.5f}"


@pytest.mark.parametrize("model,ksplit", [("qwen2-0.5b", "1"), ("qwen2-0.5b", "2"), ("tiny-hd64", "8")])
def test_int8_step_kernel_split_k_down(monkeypatch, model, ksplit):
    """Split inputs through the step kernel on every prompt token, against the oracle's logits: the
    0.5B shape's down projection unsplit and over two CTAs (the second CTA's row partials handed to
    the first as tagged words; the default), and the tiny model's down projection forced over four
    CTAs (three partners' partials; by default only inputs of 16,384 or more are split four ways)."""
    from seedplane_b200.engine import CudaQwen2
    monkeypatch.setenv("SEEDPLANE_PREFILL", "steps")
    monkeypatch.setenv("SEEDPLANE_STEP_KSPLIT", ksplit)
    cfg = PRESETS[model]
    w = make_int8_blockwise(cfg, seed=1)
    prompt = random_prompt(cfg.vocab, 6, seed=4)
    eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
    kv = eng.new_kv(32)
    stepped, _ = eng.forward(kv, prompt, all_logits=True)
    eng.close()
    want, _ = OracleQwen2(cfg, w, kv_fp16=True).forward(prompt, None, all_logits=True)
    assert_logits_close(stepped, want)


def test_int8_prompt_through_step_kernel_matches_batched(monkeypatch):
    """The same prompt through the step kernel (one launch per token) and through the batched pass."""
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS["tiny-untied"]
    w = make_int8_blockwise(cfg, seed=3, std=0.1)
    prompt = random_prompt(cfg.vocab, 11, seed=2)
    eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
    kv = eng.new_kv(32)
    batched, _ = eng.forward(kv, prompt, all_logits=True)
    eng.close()
    monkeypatch.setenv("SEEDPLANE_PREFILL", "steps")
    eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
    kv = eng.new_kv(32)
    stepped, _ = eng.forward(kv, prompt, all_logits=True)
    eng.close()
    want, _ = OracleQwen2(cfg, w, kv_fp16=True).forward(prompt, None, all_logits=True)
    assert_logits_close(batched, want)
    assert_logits_close(stepped, want)


@pytest.mark.slow
def test_int8_7b_shape_long_context_decode(monkeypatch):
    """cfg5's long context on the 7B int8 shape (hidden 3584, 28 q / 4 kv heads, untied int8 LM
    head), truncated to one layer so the CPU oracle finishes: a 4,100-token prompt, then 8 greedy
    step-kernel tokens at contexts 4,100-4,107 with the attention items the kernel picks itself
    (no chunk cap), once with per-head items (28 heads x 5 chunks of ~820 positions, many
    sub-chunks per item) and once with grouped items (4 kv heads x 37 chunks, all 7 q heads of a
    group on the tensor cores). Tokens equal the oracle's; the last step's logits within the int8
    tolerance."""
    from dataclasses import replace
    from seedplane_b200.config import QWEN2_5_7B
    from seedplane_b200.engine import CudaQwen2
    cfg = replace(QWEN2_5_7B, layers=1, max_positions=8192, name="qwen2.5-7b-1l")
    w = make_int8_blockwise(cfg, seed=0, std=0.02)
    prompt = random_prompt(cfg.vocab, 4100, seed=0)
    runs = []
    for group_ctx in (str(1 << 30), "0"):
        monkeypatch.setenv("SEEDPLANE_ATTN_GROUP_CTX", group_ctx)
        eng = CudaQwen2(cfg, w, device="cuda:0", weight_format="i8")
        kv = eng.new_kv(4160)
        _, argmax = eng.forward(kv, prompt, want_logits=False)
        first = int(argmax[-1])
        toks, logits = eng.decode(kv, first, len(prompt), 8, want_logits=True)
        runs.append(([first] + toks.cpu().tolist(), logits.float().cpu()))
        eng.status()
        eng.close()
    o = OracleQwen2(cfg, w, kv_fp16=True)
    del w
    cache = o.new_cache(4160)
    lg, cache = o.forward(prompt, cache)
    want, margins = [int(lg[-1].argmax())], []
    for i in range(8):
        top = torch.topk(lg[-1], 2).values
        margins.append(float(top[0] - top[1]))
        lg, cache = o.forward([want[-1]], cache)
        if i < 7:
            want.append(int(lg[-1].argmax()))
    # the engine's last step produced the logits after token got[7] (= want[7] when all match)
    for got, logits in runs:
        assert got[:8] == want[:8], (got, want, margins)
        assert_logits_close(logits, lg[-1])
