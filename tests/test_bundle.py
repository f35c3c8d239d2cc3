"""seedplane-bundle/2 loading (`seedplane_b200.bundle.load_bundle_v2`) on bundles written by the
reference's converter (`seedplane/native_bundle.py:62-137`).

The manifests under tests/golden/ were written by the reference's own `convert` for seeded
checkpoints (tests/golden/make_bundle_golden.py); `bundle_fixture.rebuild` reproduces the weights
blob byte for byte (checked against the converter's SHA-256) before anything loads it.

CPU: architecture, plan and every tensor of the tiny bundle against the checkpoint it came from,
the sha256 check of the loader, and `load_checkpoint`'s format dispatch. GPU: the Qwen2-0.5B
bundle through `NativeEngine` and `Qwen2Engine` gives the tokens the reference itself produced for
that checkpoint (tests/golden/qwen2-0.5b.json), and the same tokens as the HF directory.
"""
import json

import pytest
import torch

import bundle_fixture
from seedplane_b200.config import PRESETS, QWEN2_0_5B
from seedplane_b200.randinit import TEST_INIT, make_weights


@pytest.fixture(scope="module")
def tiny_bundle(tmp_path_factory):
    cfg = PRESETS["tiny-hd64"]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    d = bundle_fixture.rebuild("tiny-hd64", w, cfg, tmp_path_factory.mktemp("bundle") / "tiny.sp")
    return cfg, w, d


def test_tiny_bundle_arch_plan_and_tensors(tiny_bundle):
    from seedplane_b200.bundle import load_bundle_v2, load_checkpoint, plan_of
    cfg, w, d = tiny_bundle
    got_cfg, t, fmt = load_bundle_v2(d, verify_sha256=True)
    assert fmt == "f16"
    for field in ("layers", "hidden", "heads", "kv_heads", "intermediate", "vocab", "head_dim",
                  "tied_embeddings"):
        assert getattr(got_cfg, field) == getattr(cfg, field), field
    assert got_cfg.rope_theta == cfg.rope_theta and got_cfg.rms_norm_eps == cfg.rms_norm_eps
    assert plan_of(d) == {"shard": 64, "halo": 32, "sinks": 4}
    meta = bundle_fixture.manifest("tiny-hd64")
    assert set(t) == set(meta["tensors"])
    for key, spec in meta["tensors"].items():
        want = bundle_fixture.source_tensor(w, cfg, key).float()
        assert list(t[key].shape) == spec["shape"], key
        assert t[key].dtype == (torch.float16 if spec["dtype"] == "f16" else torch.float32), key
        assert torch.equal(t[key].float(), want), key          # fp16 weights convert exactly
    # the loader dispatches on the manifest's format
    assert load_checkpoint(d)[1].keys() == t.keys()


def test_bundle_sha256_mismatch_is_refused(tiny_bundle, tmp_path):
    import shutil
    from seedplane_b200.bundle import load_bundle_v2
    cfg, w, d = tiny_bundle
    bad = tmp_path / "bad.sp"
    shutil.copytree(d, bad)
    with open(bad / "weights.spw", "r+b") as f:
        f.seek(1000)
        b = f.read(1)
        f.seek(1000)
        f.write(bytes([b[0] ^ 1]))
    with pytest.raises(ValueError, match="sha256"):
        load_bundle_v2(bad, verify_sha256=True)


def test_rebuild_refuses_other_weights(tmp_path):
    cfg = PRESETS["tiny-hd64"]
    w = make_weights(cfg, seed=1, dtype=torch.float16, **TEST_INIT)      # not the converter's checkpoint
    with pytest.raises(ValueError, match="sha256"):
        bundle_fixture.rebuild("tiny-hd64", w, cfg, tmp_path / "x.sp")


@pytest.mark.gpu
def test_qwen2_0_5b_bundle_tokens(tmp_path, golden_dir):
    from seedplane_b200.native import NativeEngine
    from seedplane_b200.qwen_engine import Qwen2Engine
    gold = json.loads((golden_dir / "qwen2-0.5b.json").read_text())
    w = make_weights(QWEN2_0_5B, seed=0, dtype=torch.float16)
    d = bundle_fixture.rebuild("qwen2-0.5b", w, QWEN2_0_5B, tmp_path / "q05.sp")
    del w
    want = gold["fp16_weights"]["tokens"]
    with NativeEngine(d, ctx=256, max_new_tokens=32) as ne:
        list(ne.generate(ids=gold["prompt"], temperature=0.0))
        assert ne.last_tokens[:32] == want
        assert ne.info["plan"] == {"shard": 512, "halo": 256, "sinks": 4}
    e = Qwen2Engine(d)
    cache = e.new_cache(128)
    logits, cache = e.forward(gold["prompt"], cache)
    toks = [int(logits[-1].argmax())]
    for _ in range(31):
        logits, cache = e.forward([toks[-1]], cache)
        toks.append(int(logits[-1].argmax()))
    assert toks == want
