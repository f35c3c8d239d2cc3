"""Top-k / top-p filtering on the device (`sp_sample_filter`) against the kept sets the reference's
own `Qwen2Engine.sample` produced (`tests/golden/sample_filter.json`), and draws from the filtered
row (`sample_token`): always inside the kept set, top_k = 1 is the argmax, and the frequencies of
many draws follow the renormalized softmax."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.speculative_oracle import sample_filter as oracle_filter
from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights

pytestmark = pytest.mark.gpu
GOLDEN = json.loads((Path(__file__).parent / "golden" / "sample_filter.json").read_text())["cases"]


def logits_row(seed, V, scale):
    return np.random.default_rng(seed).standard_normal(V).astype(np.float32) * np.float32(scale)


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"s{c['seed']}-V{c['V']}-T{c['temperature']}-k{c['top_k']}-p{c['top_p']}")
def test_device_filter_matches_reference_kept_set(case):
    from seedplane_b200.speculative import sample_filter
    l = logits_row(case["seed"], case["V"], case["scale"])
    z = sample_filter(torch.from_numpy(l).cuda(), case["temperature"], case["top_k"], case["top_p"])
    z = z.cpu().numpy()[0]
    kept = np.flatnonzero(np.isfinite(z))
    assert kept.tolist() == case["kept"]
    want = (l / np.float32(case["temperature"])).astype(np.float32)
    assert np.array_equal(z[kept], want[kept])           # z = logits / T, the fp32 division
    assert np.array_equal(np.isfinite(oracle_filter(l, case["temperature"], case["top_k"], case["top_p"])),
                          np.isfinite(z))


@pytest.fixture(scope="module")
def engine():
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS["tiny-hd64"]
    eng = CudaQwen2(cfg, make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT), device="cuda:0")
    yield eng
    eng.close()


def test_filtered_draws(engine):
    from seedplane_b200.speculative import sample_token
    l = logits_row(5, 1000, 3.0)
    row = torch.from_numpy(l).cuda()
    for T, k, p in [(1.0, 20, 1.0), (0.8, 0, 0.9), (1.5, 50, 0.8)]:
        kept = set(np.flatnonzero(np.isfinite(oracle_filter(l, T, k, p))).tolist())
        got = {sample_token(engine, row, T, 9, c, k, p) for c in range(200)}
        assert got <= kept and len(got) > 1
    am = int(np.argmax(l))
    assert all(sample_token(engine, row, 2.0, 3, c, 1, 1.0) == am for c in range(20))
    # frequencies of 4,000 draws against softmax over the top 5 (loose: 4 sigma)
    z = oracle_filter(l, 1.0, 5, 1.0).astype(np.float64)
    idx = np.flatnonzero(np.isfinite(z))
    p = np.exp(z[idx] - z[idx].max())
    p /= p.sum()
    n = 4000
    draws = np.array([sample_token(engine, row, 1.0, 21, c, 5, 1.0) for c in range(n)])
    freq = np.array([(draws == i).sum() for i in idx]) / n
    assert np.all(np.abs(freq - p) <= 4 * np.sqrt(p * (1 - p) / n) + 1e-3)


def test_filter_rejects_bad_arguments():
    from seedplane_b200.speculative import sample_filter
    row = torch.zeros(100, device="cuda:0")
    for T, k, p in [(0.0, 0, 0.9), (1.0, -1, 0.9), (1.0, 0, 1.5), (1.0, 0, -0.1)]:
        with pytest.raises(ValueError):
            sample_filter(row, T, k, p)
