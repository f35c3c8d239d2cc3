"""Token identity of the CUDA engine with the oracle on the benchmark architectures.

* Qwen2-0.5B (the reference's own CPU configuration shape): fp16-rounded random-init weights,
  64-token prompt, 32 greedy tokens; also compared with the golden tokens the reference produced.
* Qwen2-1.5B (the headline configuration): 512-token prompt, 256 greedy tokens, 4096-slot cache.
"""
import json

import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import QWEN2_0_5B, QWEN2_1_5B
from seedplane_b200.randinit import make_weights, random_prompt

pytestmark = pytest.mark.gpu


def _engine_greedy(eng, prompt, n, capacity):
    kv = eng.new_kv(capacity)
    _, argmax = eng.forward(kv, prompt, want_logits=False)
    first = int(argmax[-1])
    out, _ = eng.decode(kv, first, len(prompt), n - 1)
    eng.status()
    return [first] + out.cpu().tolist()


def _first_divergence(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def test_qwen2_0_5b_greedy_tokens(golden_dir):
    from seedplane_b200.engine import CudaQwen2
    torch.set_num_threads(max(1, torch.get_num_threads()))
    gold = json.loads((golden_dir / "qwen2-0.5b.json").read_text())
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    eng = CudaQwen2(QWEN2_0_5B, w)
    got = _engine_greedy(eng, gold["prompt"], 32, 96)
    want, margins = OracleQwen2(QWEN2_0_5B, w, kv_fp16=True).greedy(gold["prompt"], 32)
    assert got == want, (_first_divergence(got, want), margins)
    # the reference itself (fp32 K/V) gives the same tokens on this checkpoint
    assert got == gold["fp16_weights"]["tokens"]
    eng.close()


@pytest.mark.slow
def test_qwen2_1_5b_greedy_512_plus_256():
    from seedplane_b200.engine import CudaQwen2
    w = make_weights(QWEN2_1_5B, seed=0, dtype=torch.float16)
    prompt = random_prompt(QWEN2_1_5B.vocab, 512, seed=0)
    eng = CudaQwen2(QWEN2_1_5B, w)
    got = _engine_greedy(eng, prompt, 256, 4096)
    eng.close()
    want, margins = OracleQwen2(QWEN2_1_5B, w, kv_fp16=True).greedy(prompt, 256)
    d = _first_divergence(got, want)
    assert d is None, f"first divergence at {d}: margin there {margins[d]:.5f}, min margin {min(margins):.5f}"


@pytest.mark.parametrize("gemv", ["tc", "hmma"])
def test_chain_path_greedy_tokens(golden_dir, monkeypatch, gemv):
    """The kernel-per-op decode chain (SEEDPLANE_STEP=chain: one GEMV launch per projection, the
    standalone decode attention kernel; SEEDPLANE_GEMV=hmma: its mma.sync GEMV instead of the
    tcgen05 one) gives the oracle's tokens on the Qwen2-0.5B shape, like the persistent step kernel."""
    from seedplane_b200.engine import CudaQwen2
    gold = json.loads((golden_dir / "qwen2-0.5b.json").read_text())
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    monkeypatch.setenv("SEEDPLANE_STEP", "chain")
    if gemv == "hmma":
        monkeypatch.setenv("SEEDPLANE_GEMV", "hmma")
    eng = CudaQwen2(QWEN2_0_5B, w)        # the switches are read when the engine is created
    got = _engine_greedy(eng, gold["prompt"], 32, 96)
    eng.close()
    assert got == gold["fp16_weights"]["tokens"], _first_divergence(got, gold["fp16_weights"]["tokens"])
