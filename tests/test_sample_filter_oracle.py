"""The CPU restatement of the reference's top-k / top-p masking (`oracle.speculative_oracle.
sample_filter`) against the kept sets the reference's own `Qwen2Engine.sample` produced
(`tests/golden/sample_filter.json`, made by `tests/golden/make_sample_filter_golden.py`)."""
import json
from pathlib import Path

import numpy as np

from oracle.speculative_oracle import sample_filter

GOLDEN = json.loads((Path(__file__).parent / "golden" / "sample_filter.json").read_text())["cases"]


def test_oracle_filter_matches_reference_golden():
    assert len(GOLDEN) >= 30
    for c in GOLDEN:
        l = np.random.default_rng(c["seed"]).standard_normal(c["V"]).astype(np.float32) * np.float32(c["scale"])
        z = sample_filter(l, c["temperature"], c["top_k"], c["top_p"])
        assert np.flatnonzero(np.isfinite(z)).tolist() == c["kept"], c
