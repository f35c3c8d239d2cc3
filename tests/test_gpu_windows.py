"""Shard-window attention on the GPU: every session mode of the B200 engine against tokens the
reference produced under its window definition (`tests/golden/windows.json`: `seedplane/engine.py`
ShardPlan + `Qwen2Engine` with fp16-rounded weights, recomputed per position as
`experiments/v19/oracle_windows.py` does), the approximate reuse mode against the oracle's
restatement of the native session (`qwen_vk.cpp:518-565`), window K/V copies, and NativeEngine
decoding a SeedPlane bundle under its plan."""
import json

import pytest
import torch

from oracle import window_oracle as wo
from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS, QWEN2_0_5B
from seedplane_b200.randinit import TEST_INIT, make_weights, random_prompt
from seedplane_b200.windows import MODES, ShardPlan, WindowSession

pytestmark = pytest.mark.gpu

EXACT = ("rebuild", "rebuild-batch", "shadow", "shadow-batch")


def _cases(golden_dir, model):
    cases = json.loads((golden_dir / "windows.json").read_text())["cases"]
    return [c for c in cases if c["model"] == model and c["weights"] == "fp16"]


def _session_greedy(eng, mode, plan, prompt, n, positions=None, block=32):
    """Greedy tokens of a WindowSession: batched catch-up, then device decode blocks."""
    s = WindowSession(eng, mode, ShardPlan(**plan), positions)
    try:
        s.seq.extend(prompt)
        _, t = s.catch_up()
        out = [t]
        while len(out) < n:
            s.seq.append(out[-1])
            got, _ = s.decode_block(min(block, n - len(out)))
            got = got.tolist()
            out += got
            s.seq.extend(got[:-1])
            s.commit_block(len(got))
        return out[:n]
    finally:
        s.close()


@pytest.fixture(scope="module")
def tiny_engines():
    from seedplane_b200.engine import CudaQwen2
    out = {}
    for name in ("tiny-hd64", "tiny-hd128"):
        cfg = PRESETS[name]
        w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
        out[name] = (CudaQwen2(cfg, w), cfg, w)
    yield out
    for eng, _, _ in out.values():
        eng.close()


@pytest.mark.parametrize("mode", EXACT)
@pytest.mark.parametrize("model", ["tiny-hd64", "tiny-hd128"])
def test_exact_modes_give_the_reference_window_tokens(golden_dir, tiny_engines, model, mode):
    eng, cfg, w = tiny_engines[model]
    for c in _cases(golden_dir, model):
        p = c["plan"]
        got = _session_greedy(eng, mode, p, c["prompt"], len(c["tokens"]))
        assert got == c["tokens"], (mode, p)
        # short blocks: more window moves fall between device blocks
        assert _session_greedy(eng, mode, p, c["prompt"], len(c["tokens"]), block=5) == c["tokens"], (mode, p)


@pytest.mark.parametrize("model", ["tiny-hd64", "tiny-hd128"])
def test_reuse_and_full_modes_match_the_oracle_session(tiny_engines, model):
    eng, cfg, w = tiny_engines[model]
    oracle = OracleQwen2(cfg, w, kv_fp16=True)
    prompt = random_prompt(cfg.vocab, 21, seed=3)
    for mode, plan in (("reuse", (16, 8, 4)), ("reuse", (12, 12, 2)), ("reuse", (10, 0, 0)), ("full", (16, 8, 4))):
        want, why = wo.session_greedy(oracle, prompt, 50, mode, *plan, positions=cfg.max_positions)
        assert why == "length"
        got = _session_greedy(eng, mode, dict(zip(("shard", "halo", "sinks"), plan)), prompt, 50)
        assert got == want, (mode, plan)


def test_every_mode_on_a_prompt_that_spans_many_windows(tiny_engines):
    """A 70-token prompt over 12-token shards goes through the batched pass window by window; the
    exact modes agree with the window definition, reuse with the oracle session."""
    eng, cfg, w = tiny_engines["tiny-hd64"]
    oracle = OracleQwen2(cfg, w, kv_fp16=True)
    prompt = random_prompt(cfg.vocab, 70, seed=11)
    exact = wo.window_greedy(oracle, prompt, 30, 12, 6, 3)
    for mode in MODES:
        plan = {"shard": 12, "halo": 6, "sinks": 3}
        got = _session_greedy(eng, mode, plan, prompt, 30, positions=512)
        if mode in EXACT:
            assert got == exact, mode
        else:
            want, _ = wo.session_greedy(oracle, prompt, 30, mode, 12, 6, 3, positions=512)
            assert got == want, mode


def test_qwen2_0_5b_shadow_batch_gives_the_reference_window_tokens(golden_dir):
    """The Qwen2-0.5B shape (fp16 weights, 64-token prompt, 40 tokens over 32-token shards with a
    16-token halo and 4 sinks) in the default mode and in rebuild-batch."""
    from seedplane_b200.engine import CudaQwen2
    c = _cases(golden_dir, "qwen2-0.5b")[0]
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    eng = CudaQwen2(QWEN2_0_5B, w)
    try:
        for mode in ("shadow-batch", "rebuild-batch"):
            assert _session_greedy(eng, mode, c["plan"], c["prompt"], len(c["tokens"])) == c["tokens"], mode
    finally:
        eng.close()


def test_kv_copy_moves_slots_between_caches(tiny_engines):
    """A window seeded by sp_kv_copy continues exactly like the cache it was copied from; bad
    ranges are rejected before any copy."""
    eng, cfg, w = tiny_engines["tiny-hd128"]
    a, b = eng.new_kv(40), eng.new_kv(64)
    try:
        prompt = random_prompt(cfg.vocab, 30, seed=1)
        _, am = eng.forward(a, prompt, want_logits=False)
        eng.kv_copy(a, 0, b, 0, 30)
        b.length = 30
        t = int(am[-1])
        ta, _ = eng.decode(a, t, 30, 8)
        tb, _ = eng.decode(b, t, 30, 8)
        assert ta.tolist() == tb.tolist()
        with pytest.raises(Exception):
            eng.kv_copy(a, 30, b, 0, 20)     # past the source capacity
        with pytest.raises(Exception):
            eng.kv_copy(a, 0, a, 2, 4)       # overlapping ranges in one cache
    finally:
        a.close()
        b.close()


def test_native_engine_decodes_a_bundle_under_its_plan(golden_dir, tmp_path):
    """A SeedPlane bundle whose seedplane.json carries a plan: NativeEngine defaults to shadow-batch
    under it (as the reference engine does), `--shard/--halo/--sinks` override it, `full=True`
    turns windows off; info reports mode, plan, positions and window slots."""
    from safetensors.torch import save_file
    from seedplane_b200.native import NativeEngine
    c = [x for x in _cases(golden_dir, "tiny-hd128") if x["plan"]["shard"] == 16][0]
    cfg = PRESETS["tiny-hd128"]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    (tmp_path / "config.json").write_text(json.dumps(cfg.to_hf()))
    save_file({k: v.contiguous() for k, v in w.items()}, str(tmp_path / "model.safetensors"))
    (tmp_path / "seedplane.json").write_text(json.dumps({"plan": c["plan"]}))
    with NativeEngine(tmp_path) as eng:
        p = c["plan"]
        assert eng.info["mode"] == "shadow-batch" and eng.info["plan"] == p
        assert eng.info["positions"] == cfg.max_positions
        assert eng.info["window_slots"] == p["shard"] + p["halo"] + p["sinks"]
        list(eng.generate(ids=c["prompt"], max_new_tokens=len(c["tokens"])))
        assert eng.last_tokens == c["tokens"]
        # a continuation request crosses more boundaries: each new token is its window's argmax
        more = random_prompt(cfg.vocab, 5, seed=2)
        list(eng.generate(ids=more, reset=False, max_new_tokens=20))
        seq = eng.state()["tokens"]
        oracle = OracleQwen2(cfg, w, kv_fp16=True)
        vis = wo.visible_indices(len(seq), p["shard"], p["halo"], p["sinks"])
        for j in range(len(seq) - 20, len(seq)):
            idx = vis[j - 1]
            logits, _ = oracle.forward([seq[i] for i in idx], oracle.new_cache(len(idx)), positions=idx)
            assert seq[j] == int(logits[-1].argmax()), j
    c2 = [x for x in _cases(golden_dir, "tiny-hd128") if x["plan"]["shard"] == 24][0]
    with NativeEngine(tmp_path, mode="rebuild", extra_args=("--shard", "24", "--halo", "4", "--sinks", "1")) as eng:
        assert eng.info["mode"] == "rebuild" and eng.info["plan"] == c2["plan"]
        list(eng.generate(ids=c2["prompt"], max_new_tokens=len(c2["tokens"])))
        assert eng.last_tokens == c2["tokens"]
    with NativeEngine(tmp_path, full=True, ctx=300) as eng:
        assert eng.info["mode"] == "full" and eng.info["positions"] == 300 and eng.info["window_slots"] == 300
        assert eng.info["plan"] == {"shard": 300, "halo": 0, "sinks": 0}
