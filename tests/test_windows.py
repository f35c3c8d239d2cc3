"""Shard-window attention on the CPU: the window oracle pinned on tokens the reference itself produced
(`tests/golden/windows.json`, made by `make_window_golden.py` from `seedplane/engine.py`'s ShardPlan
and `Qwen2Engine`), the oracle's session modes against the window definition, and the product's
`WindowSession` / `NativeEngine` host logic against the oracle over a context-sensitive fake model
(each K/V slot remembers the context it was computed in, so a window move that keeps stale or
misplaced K/V changes later tokens)."""
import json

import pytest
import torch

from oracle import window_oracle as wo
from oracle.qwen_oracle import OracleQwen2
from seedplane_b200 import native as nat
from seedplane_b200.config import PRESETS, QWEN2_0_5B
from seedplane_b200.randinit import make_weights
from seedplane_b200.windows import MODES, ShardPlan, WindowSession

V = 101
EXACT = ("rebuild", "rebuild-batch", "shadow", "shadow-batch")


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "windows.json").read_text())["cases"]


def _model(case):
    cfg = PRESETS.get(case["model"], QWEN2_0_5B)
    dtype = torch.float16 if case["weights"] == "fp16" else torch.float32
    w = make_weights(cfg, seed=0, dtype=dtype, **case["init"])
    return OracleQwen2(cfg, w, kv_fp16=case["kv_fp16"])


# ---- the oracle against the reference ------------------------------------------------------------

def test_window_indices_match_the_reference_window_sizes(golden):
    for c in golden:
        p = c["plan"]
        total = len(c["prompt"]) + len(c["tokens"])
        vis = wo.visible_indices(total, p["shard"], p["halo"], p["sinks"])
        for i, n in c["window_sizes"].items():
            assert len(vis[int(i)]) == n and vis[int(i)][-1] == int(i)
        ours = ShardPlan(**p)
        for (a0, a1, ai), (b0, b1, bi) in zip(ours.windows(total), wo.windows(total, **p)):
            assert (a0, a1, ai.tolist()) == (b0, b1, bi)


@pytest.mark.parametrize("which", range(9))
def test_window_oracle_matches_the_reference_tiny(golden, which):
    c = [g for g in golden if g["model"].startswith("tiny")][which]
    m = _model(c)
    p = c["plan"]
    assert wo.window_greedy(m, c["prompt"], len(c["tokens"]), p["shard"], p["halo"], p["sinks"]) == c["tokens"]


def test_window_oracle_matches_the_reference_qwen2_0_5b(golden):
    c = [g for g in golden if g["model"] == "qwen2-0.5b"][0]
    m = _model(c)
    p = c["plan"]
    assert wo.window_greedy(m, c["prompt"], len(c["tokens"]), p["shard"], p["halo"], p["sinks"]) == c["tokens"]


@pytest.mark.parametrize("mode", EXACT)
def test_oracle_session_exact_modes_give_the_window_tokens(golden, mode):
    """The native session's exact modes (qwen_vk.cpp:518-565) reproduce the window definition."""
    for c in [g for g in golden if g["model"].startswith("tiny")][:6]:
        p = c["plan"]
        if mode not in ("rebuild", "rebuild-batch") and (p["halo"] > p["shard"] or p["sinks"] > p["shard"]):
            continue
        toks, reason = wo.session_greedy(_model(c), c["prompt"], len(c["tokens"]), mode, p["shard"], p["halo"],
                                         p["sinks"], 4096)
        assert reason == "length" and toks == c["tokens"], (mode, p)


# ---- the product's session logic over a fake model -------------------------------------------------

def _state(token, pos, ctx):
    """A slot's K/V stand-in: depends on the token, its position and every visible slot before it."""
    h = (int(token) * 1000003 + int(pos) * 7919) % (1 << 31)
    for k, c in enumerate(ctx):
        h = (h * 131 + int(c) * (k + 3)) % (1 << 31)
    return h


class FakeKV:
    def __init__(self, capacity):
        self.capacity, self.length, self.slots = capacity, 0, [None] * capacity

    def close(self):
        pass


class FakeEngine:
    """The engine calls the session makes (forward / decode at kv.length, kv_copy)."""
    device = torch.device("cpu")

    def __init__(self, max_positions=4096):
        self.cfg = type("C", (), {"vocab": V, "max_positions": max_positions})()
        self.calls = []

    def new_kv(self, capacity):
        return FakeKV(capacity)

    def kv_copy(self, src, s0, dst, d0, n):
        assert s0 + n <= src.capacity and d0 + n <= dst.capacity and None not in src.slots[s0:s0 + n]
        dst.slots[d0:d0 + n] = src.slots[s0:s0 + n]

    def forward(self, kv, ids, positions=None, want_logits=False, last_only=False):
        ids = [int(t) for t in ids]
        pos = list(positions) if positions is not None else list(range(kv.length, kv.length + len(ids)))
        self.calls.append(("forward", len(ids)))
        out = []
        for t, p in zip(ids, pos):
            s = kv.length
            assert s < kv.capacity, "window overflow"
            kv.slots[s] = _state(t, p, kv.slots[:s])
            kv.length = s + 1
            out.append(kv.slots[s] % V)
        logits = torch.nn.functional.one_hot(torch.tensor(out[-1:]), V).float() if want_logits else None
        return logits, torch.tensor(out)

    def decode(self, kv, token, pos, n, want_logits=False):
        out = []
        for k in range(n):
            _, am = self.forward(kv, [token], [pos + k])
            token = int(am[-1])
            out.append(token)
        return torch.tensor(out), (torch.nn.functional.one_hot(torch.tensor(out[-1]), V).float() if want_logits
                                   else None)


class FakeOracleCache:
    def __init__(self, capacity):
        self.keys = [torch.full((capacity,), -1, dtype=torch.int64)]
        self.values = [torch.zeros(capacity, dtype=torch.int64)]
        self.length, self.capacity = 0, capacity


class FakeOracleModel:
    """The same stand-in behind the oracle's model interface (OracleQwen2.forward / new_cache)."""

    def new_cache(self, capacity):
        return FakeOracleCache(capacity)

    def forward(self, ids, cache, positions=None, slots=None, advance=True, all_logits=False):
        ids = [int(t) for t in ids]
        slots = list(slots) if slots is not None else list(range(cache.length, cache.length + len(ids)))
        pos = list(positions) if positions is not None else slots
        last = None
        for t, p, s in zip(ids, pos, slots):
            ctx = cache.keys[0][:s].tolist()
            assert -1 not in ctx, "a visible slot was never written"
            cache.keys[0][s] = _state(t, p, ctx)
            last = int(cache.keys[0][s]) % V
        if advance:
            cache.length = max(cache.length, slots[-1] + 1)
        return torch.nn.functional.one_hot(torch.tensor([last]), V).float(), cache


PLANS = [(8, 4, 2), (8, 0, 0), (6, 6, 3), (7, 3, 0), (5, 2, 7), (9, 1, 9)]


def _valid(mode, plan):
    s, h, k = plan
    return mode in ("full", "rebuild", "rebuild-batch") or (h <= s and k <= s)


@pytest.mark.parametrize("mode", MODES)
def test_session_matches_the_oracle_session(mode):
    """WindowSession (batched catch-up, device-style decode blocks, window moves) gives the
    oracle session's tokens for every mode, prompts that cross several boundaries included."""
    for plan in PLANS:
        if not _valid(mode, plan):
            with pytest.raises(ValueError):
                WindowSession(FakeEngine(), mode, ShardPlan(*plan), 64)
            continue
        for n_prompt in (1, 5, 19):
            prompt = [(7 * i + 3) % V for i in range(n_prompt)]
            want, why = wo.session_greedy(FakeOracleModel(), prompt, 50, mode, *plan, positions=60)
            eng = FakeEngine()
            s = WindowSession(eng, mode, ShardPlan(*plan), 60)
            s.seq.extend(prompt)
            _, t = s.catch_up()
            got = [t]
            try:
                while len(got) < 50:
                    s.seq.append(got[-1])
                    out, _ = s.decode_block(min(4, 50 - len(got)))
                    got += out.tolist()
                    s.seq.extend(out.tolist()[:-1])
                    s.commit_block(len(out))
            except RuntimeError as exc:
                assert str(exc).startswith("context full")
            if why == "context":
                assert got[:len(want)] == want, (mode, plan, n_prompt)
            else:
                assert got[:50] == want, (mode, plan, n_prompt)


def _window_argmax(seq, i, plan):
    vis = wo.visible_indices(len(seq), *plan)[i]
    logits, _ = FakeOracleModel().forward([seq[j] for j in vis], FakeOracleCache(len(vis)), positions=vis)
    return int(logits[-1].argmax())


@pytest.mark.parametrize("mode", EXACT + ("full",))
def test_native_engine_runs_follow_the_window_definition(mode):
    """NativeEngine runs (device blocks of 32 cut at stop tokens, continuation requests, reset) in
    an exact mode: every sampled token is the argmax of its position's window."""
    plan = (16, 8, 4) if mode != "full" else (60, 0, 0)
    eng = nat.NativeEngine.__new__(nat.NativeEngine)
    eng.cfg = type("C", (), {"vocab": V})()
    eng._engine, eng._tok = FakeEngine(), None
    eng._session = WindowSession(eng._engine, mode, ShardPlan(*plan), 120)
    eng.capacity = 120
    eng._stop_ids = set()
    eng.defaults = {"temperature": None, "top_k": None, "top_p": None, "seed": None, "max_new_tokens": 256}
    eng.system, eng.last, eng.last_tokens, eng.on_token, eng.bundle = nat.DEFAULT_SYSTEM, None, [], None, "fake"
    for reset, ids, kw in ((True, [5, 9, 2], {"max_new_tokens": 30}),
                           (False, [11, 4], {"max_new_tokens": 40, "stop": []}),
                           (False, [1] * 3, {"max_new_tokens": 25})):
        before = len(eng._history) if not reset else 0
        list(eng.generate(ids=ids, reset=reset, **kw))
        seq = eng._history
        start = before + len(ids)
        assert eng.last_tokens == seq[start:]
        for j in range(start, len(seq)):
            assert seq[j] == _window_argmax(seq, j - 1, plan if mode != "full" else (1000, 0, 0)), (mode, j)
        assert eng.state()["processed"] == len(seq) - 1
    # a stop token cuts a device block: the next request continues from the kept tokens
    list(eng.generate(ids=[3, 3], reset=True, max_new_tokens=40))
    full_run = list(eng.last_tokens)
    stop = full_run[20]
    list(eng.generate(ids=[3, 3], reset=True, max_new_tokens=40, stop=[stop]))
    k = full_run.index(stop)
    assert eng.last_tokens == full_run[:k + 1] and eng.last["reason"] == "stop"
    list(eng.generate(ids=[8], reset=False, max_new_tokens=10))
    seq = eng._history
    for j in range(len(seq) - 10, len(seq)):
        assert seq[j] == _window_argmax(seq, j - 1, plan if mode != "full" else (1000, 0, 0))


def test_context_full_ends_the_run():
    eng = FakeEngine()
    s = WindowSession(eng, "shadow-batch", ShardPlan(8, 4, 2), 20)
    s.seq.extend(range(1, 20))
    s.catch_up()
    s.seq.append(7)
    out, _ = s.decode_block(10)
    assert len(out) == 1                   # position 19 is the last one
    s.seq.append(int(out[-1]))
    s.commit_block(1)
    with pytest.raises(RuntimeError, match="context full"):
        s.decode_block(1)


def test_shard_plan_validation_matches_the_reference():
    for kw, msg in (({"shard": 0}, "shard must be greater than zero"), ({"halo": -1}, "halo must be non-negative"),
                    ({"sinks": -1}, "sinks must be non-negative")):
        with pytest.raises(ValueError, match=msg):
            ShardPlan(**kw)
    with pytest.raises(ValueError, match="sequence length"):
        list(ShardPlan().windows(-1))
    assert list(ShardPlan().windows(0)) == []
