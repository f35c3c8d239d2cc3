"""The stochastic acceptance oracle on the CPU (no reference counterpart: parity unpinned; these
pin its own arithmetic and the rule's basic behaviour)."""
import math

import numpy as np

from oracle.speculative_oracle import accept_stochastic, dexp_ref


def test_dexp_matches_exp():
    x = np.linspace(-700.0, 0.0, 20001)          # normal results (below ~-708 they are subnormal)
    got = dexp_ref(x)
    want = np.array([math.exp(v) for v in x])
    rel = np.abs(got - want) / want
    assert float(rel.max()) < 1e-15
    assert dexp_ref(np.array([-800.0]))[0] == 0.0


def test_identical_drafter_always_accepts():
    rng = np.random.default_rng(0)
    V = 50
    logits = rng.normal(size=(3, V)).astype(np.float32)
    toks, pars = [int(np.argmax(logits[0])), 7], [-1, 0]
    for seed in range(20):
        emitted, acc = accept_stochastic(toks, pars, logits, logits, 1.0, seed, 0)
        assert acc == [0, 1] and emitted == toks           # p / q = 1 > u: every draft accepted


def test_rootless_draw_follows_the_target():
    V = 6
    logits = np.log(np.array([[0.5, 0.2, 0.1, 0.1, 0.05, 0.05]], dtype=np.float64)).astype(np.float32)
    counts = np.zeros(V)
    trials = 3000
    for c in range(trials):
        emitted, acc = accept_stochastic([], [], logits, logits, 1.0, 12345, c)
        assert acc == [] and len(emitted) == 1
        counts[emitted[0]] += 1
    p = np.exp(logits[0].astype(np.float64))
    p /= p.sum()
    assert np.all(np.abs(counts / trials - p) < 4 * np.sqrt(p * (1 - p) / trials) + 1e-3)


def test_reproducible_and_counter_dependent():
    rng = np.random.default_rng(1)
    V = 300
    t = rng.normal(size=(5, V)).astype(np.float32)
    d = rng.normal(size=(5, V)).astype(np.float32)
    toks, pars = [3, 9, 11, 4], [-1, 0, 0, 1]
    a = accept_stochastic(toks, pars, t, d, 0.8, 7, 3)
    assert a == accept_stochastic(toks, pars, t, d, 0.8, 7, 3)
    outs = {tuple(accept_stochastic(toks, pars, t, d, 0.8, 7, c)[0]) for c in range(30)}
    assert len(outs) > 1
