"""The step kernel's attention items at contexts long enough for several sub-chunks per item.

The step kernel splits a layer's attention into (q head, context chunk) items on the last CTAs,
each walking its chunk in 48-position sub-chunks. Capping the chunks per head
(`SEEDPLANE_ATTN_MAX_CHUNKS=2`) makes every item walk several sub-chunks at small contexts, with the
step's own K/V row in a later sub-chunk: the pipelined K/V staging and the row taken from the
QKV projection's hand-off words are exercised. Bars: greedy tokens identical; logits within 1e-3
of the largest |logit|.
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


@pytest.mark.parametrize("name", ["tiny-hd64", "tiny-hd128"])
def test_long_items_decode_matches_oracle(monkeypatch, name):
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[name]
    monkeypatch.setenv("SEEDPLANE_ATTN_MAX_CHUNKS", "2")
    monkeypatch.setenv("SEEDPLANE_PREFILL", "steps")        # the prompt through the step kernel too
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
