"""Record seedplane-bundle/2 manifests written by SeedPlane's own converter.

    python tests/golden/make_bundle_golden.py --reference <path to the SeedPlane source tree>

For each checkpoint below, this repository's seeded random-init weights are written as an HF
directory (fp16 safetensors + config.json) and converted by the reference's
`seedplane.native_bundle.convert` (unmodified, imported from the given tree). The manifest it
writes (`seedplane.json`: arch, plan, tensor table with offsets, SHA-256 of `weights.spw`) is kept
as `bundle_<name>.json`; the weights blob itself is not kept. A test rebuilds the blob from the
same seeded weights by the manifest's table and must reproduce the converter's SHA-256 exactly
before it loads the bundle, so the loader is exercised on byte-identical converter output.

* `tiny-hd64` (TEST_INIT, 2 layers, plan shard 64 / halo 32 / sinks 4);
* `qwen2-0.5b` (the reference's own CPU configuration shape, std 0.02, default plan).

The reference is needed only to make these files; tests read them. Run on a CPU box.
"""
from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from seedplane_b200.config import PRESETS, QWEN2_0_5B  # noqa: E402
from seedplane_b200.randinit import TEST_INIT, make_weights  # noqa: E402

CASES = {
    "tiny-hd64": (PRESETS["tiny-hd64"], TEST_INIT, {"shard": 64, "halo": 32, "sinks": 4}),
    "qwen2-0.5b": (QWEN2_0_5B, {}, {}),
}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="root of the SeedPlane source tree")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", default=None, help="one case name")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from seedplane.native_bundle import convert
    from safetensors.torch import save_file
    for name, (cfg, init, plan) in CASES.items():
        if a.only and name != a.only:
            continue
        w = make_weights(cfg, seed=0, dtype=torch.float16, **init)
        with tempfile.TemporaryDirectory() as tmp:
            src, out = Path(tmp) / "hf", Path(tmp) / "bundle"
            src.mkdir()
            (src / "config.json").write_text(json.dumps(cfg.to_hf()))
            save_file({k: v.contiguous() for k, v in w.items()}, str(src / "model.safetensors"))
            manifest = convert(src, out, **plan)
        manifest.pop("source", None)              # a temporary path
        manifest["generated_by"] = {"converter": "seedplane.native_bundle.convert", "checkpoint": name,
                                    "seed": 0, "init": init or {"std": 0.02}, "dtype": "f16"}
        (Path(a.out) / f"bundle_{name}.json").write_text(json.dumps(manifest, indent=1) + "\n")
        print(name, manifest["weights"]["sha256"])


if __name__ == "__main__":
    main()
