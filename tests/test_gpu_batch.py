"""Runtime request batching on the GPU (`sp_decode_batch`, `batch.generate_batch`): every request of
a batch gets its own greedy tokens, the same as the oracle's (`qwen_engine.py:158-166` restated) and
as decoding the request alone, with ragged prompt lengths, stop tokens ending requests inside a
device block, batches larger than one pass, and bad arguments rejected before any launch."""
import json

import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS, QWEN2_0_5B, QWEN2_1_5B
from seedplane_b200.randinit import TEST_INIT, burst_prompts, make_weights, random_prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS["tiny-hd64"]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    eng = CudaQwen2(cfg, w)
    yield eng, cfg, w
    eng.close()


def _alone(eng, prompt, n):
    kv = eng.new_kv(len(prompt) + n)
    try:
        _, am = eng.forward(kv, prompt, want_logits=False)
        first = int(am[-1])
        if n == 1:
            return [first]
        out, _ = eng.decode(kv, first, len(prompt), n - 1)
        return [first] + out.tolist()
    finally:
        kv.close()


@pytest.mark.parametrize("model", ["tiny-hd64", "tiny-hd128"])
def test_batch_matches_the_oracle_per_request(model):
    from seedplane_b200.batch import generate_batch
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS[model]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    eng = CudaQwen2(cfg, w)
    try:
        oracle = OracleQwen2(cfg, w, kv_fp16=True)
        prompts = [random_prompt(cfg.vocab, n, seed=10 + i) for i, n in enumerate((1, 5, 12, 33, 7, 64, 2, 19))]
        got = generate_batch(eng, prompts, 24, block=7)
        for p, g in zip(prompts, got):
            assert g == oracle.greedy(p, 24)[0]
        # per-request limits, and the same requests alone
        limits = [1, 3, 24, 9, 17, 2, 24, 11]
        got = generate_batch(eng, prompts, limits)
        for p, g, m in zip(prompts, got, limits):
            assert g == _alone(eng, p, m)
    finally:
        eng.close()


def test_stop_tokens_end_requests_inside_a_block(tiny):
    from seedplane_b200.batch import generate_batch
    eng, cfg, w = tiny
    prompts = [random_prompt(cfg.vocab, 9 + 3 * i, seed=40 + i) for i in range(6)]
    full = generate_batch(eng, prompts, 30)
    stop = {full[0][4], full[3][11]}
    got = generate_batch(eng, prompts, 30, stop=stop, block=8)
    for f, g in zip(full, got):
        cut = next((i for i, t in enumerate(f) if t in stop), None)
        assert g == (f if cut is None else f[:cut + 1])


def test_more_requests_than_one_pass_and_decode_batch_rows(tiny):
    from seedplane_b200.batch import MAX_BATCH, generate_batch
    eng, cfg, w = tiny
    prompts = [random_prompt(cfg.vocab, 3 + i % 11, seed=100 + i) for i in range(MAX_BATCH + 9)]
    got = generate_batch(eng, prompts, 6)
    for i in (0, 1, MAX_BATCH - 1, MAX_BATCH, MAX_BATCH + 8):
        assert got[i] == _alone(eng, prompts[i], 6), i
    # decode_batch rows: row i holds every request's token after step i
    kvs = [eng.new_kv(64) for _ in range(3)]
    try:
        firsts = []
        for kv, p in zip(kvs, prompts[:3]):
            _, am = eng.forward(kv, p, want_logits=False)
            firsts.append(int(am[-1]))
        rows = eng.decode_batch(kvs, firsts, [len(p) for p in prompts[:3]], 5).cpu().tolist()
        for j in range(3):
            assert [firsts[j]] + [rows[i][j] for i in range(5)] == _alone(eng, prompts[j], 6)
            assert kvs[j].length == len(prompts[j]) + 5
    finally:
        for kv in kvs:
            kv.close()


def test_packed_prompts_match_prompts_alone(tiny):
    """sp_prefill_batch packs whole prompts into passes of at most 512 tokens (a longer prompt runs
    alone); each request's first token and K/V equal its own prompt pass: the decode that follows
    gives the same tokens."""
    eng, cfg, w = tiny
    lens = [1, 7, 130, 3, 200, 90, 500, 17, 64]            # 130 + 200 + 90 > 512: several packs; 500 alone
    prompts = [random_prompt(cfg.vocab, n, seed=300 + i) for i, n in enumerate(lens)]
    kvs = [eng.new_kv(n + 8) for n in lens]
    try:
        firsts = eng.prefill_batch(kvs, prompts).cpu().tolist()
        assert [kv.length for kv in kvs] == lens
        for p, kv, f in zip(prompts, kvs, firsts):
            want = _alone(eng, p, 6)
            assert f == want[0]
            out, _ = eng.decode(kv, f, len(p), 5)
            assert [f] + out.cpu().tolist() == want
        with pytest.raises(Exception):
            eng.prefill_batch([kvs[0], kvs[0]], [[1], [2]])           # one cache twice
    finally:
        for kv in kvs:
            kv.close()


def test_bad_batches_are_rejected(tiny):
    eng, cfg, w = tiny
    a, b = eng.new_kv(8), eng.new_kv(8)
    try:
        with pytest.raises(Exception):
            eng.decode_batch([a, a], [1, 2], [0, 0], 1)          # one cache twice
        with pytest.raises(Exception):
            eng.decode_batch([a, b], [1, 2], [0, 0], 9)          # past the capacity
        with pytest.raises(Exception):
            eng.decode_batch([a], [cfg.vocab], [0], 1)           # token outside the vocabulary
        with pytest.raises(Exception):
            eng.decode_batch([a], [1], [cfg.max_positions], 1)   # position outside the RoPE table
        assert a.length == 0 and b.length == 0
    finally:
        a.close()
        b.close()


def test_qwen2_0_5b_batch_gives_the_reference_tokens(golden_dir):
    """The reference's cfg1 prompt (fp16-rounded weights, 32 greedy tokens) decoded inside a batch of
    five requests of other lengths."""
    from seedplane_b200.batch import generate_batch
    from seedplane_b200.engine import CudaQwen2
    gold = json.loads((golden_dir / "qwen2-0.5b.json").read_text())
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    eng = CudaQwen2(QWEN2_0_5B, w)
    try:
        prompts = [random_prompt(QWEN2_0_5B.vocab, n, seed=7 + n) for n in (17, 90, 3, 128, 600)]
        got = generate_batch(eng, [gold["prompt"]] + prompts, 32)
        assert got[0] == gold["fp16_weights"]["tokens"]
        for p, g in zip(prompts, got[1:]):                  # the 600-token prompt runs alone (> 512)
            assert g == _alone(eng, p, 32)
    finally:
        eng.close()


def test_qwen2_1_5b_burst_batch_matches_requests_alone_or_the_oracle():
    """The cfg4 burst: 16 requests (prompts 32..128 tokens) x 32 tokens as one batch on the
    Qwen2-1.5B shape (the prompts packed into batched passes, then batched decode steps). Each
    request's tokens equal the same request decoded alone (its own prompt pass, then the step
    kernel), except where the two paths part because their fp32 sums differ in order (random-init
    weights leave the two best logits very close): there the oracle decides, up to the parting token
    both equal the oracle, and at it the oracle's two best logits are a near-tie (margin < 1e-3)
    between exactly the two paths' tokens."""
    from seedplane_b200.batch import generate_batch
    from seedplane_b200.engine import CudaQwen2
    w = make_weights(QWEN2_1_5B, seed=0, dtype=torch.float16)
    eng = CudaQwen2(QWEN2_1_5B, w)
    try:
        prompts = burst_prompts(QWEN2_1_5B.vocab, 16, 32, 128, seed=0)
        got = generate_batch(eng, prompts, 32)
        alone = [_alone(eng, p, 32) for p in prompts]
    finally:
        eng.close()
    parted = [i for i in range(16) if got[i] != alone[i]]
    assert len(parted) <= 4, parted
    if parted:
        oracle = OracleQwen2(QWEN2_1_5B, w, kv_fp16=True)
        for i in parted:
            d = next(j for j in range(32) if got[i][j] != alone[i][j])
            want, _ = oracle.greedy(prompts[i], d)
            assert want == got[i][:d], i
            top = torch.topk(oracle.prefix_logits(prompts[i] + got[i][:d]), 2)
            assert float(top.values[0] - top.values[1]) < 1e-3, (i, d)
            assert {got[i][d], alone[i][d]} == set(top.indices.tolist()), (i, d)
