"""The step kernel's GEMV plans on the CPU, through the library's own host functions
(`plan_step_gemv`, `step_layout`, `step_gemv_supported`, `gemv_share`): `tests/step_plan_check.cu`
plans every GEMV of each preset shape in fp16 and in int8 the way `sp_engine_create` does and
checks that the plans are supported, the split row groups and input parts partition the matrix,
each CTA's input share fits the shared-memory layout and the packed int8 rows fit `cta_bytes`;
for the 7B int8 shape also the split choices (QKV and O two ways, down four, gate_up and the
LM head unsplit). No GPU: only host code runs."""
import shutil
import subprocess
from pathlib import Path

import pytest

from seedplane_b200.config import PRESETS

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "seedplane_b200" / "libseedplane_cuda.so"


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    assert LIB.is_file(), "build the library first: python -m seedplane_b200.build"
    exe = tmp_path_factory.mktemp("plan") / "step_plan_check"
    subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
                    f"-I{ROOT / 'include'}", f"-I{ROOT / 'seedplane_b200' / 'csrc'}",
                    str(ROOT / "tests" / "step_plan_check.cu"), "-o", str(exe), f"-L{LIB.parent}", "-lseedplane_cuda",
                    f"-Xlinker=-rpath={LIB.parent}"], check=True, capture_output=True, timeout=300)
    return exe


EXPECTED_KSPLIT = {("qwen2.5-7b", True): "2 2 1 4 1"}


@pytest.mark.parametrize("i8", [False, True], ids=["f16", "i8"])
@pytest.mark.parametrize("model", sorted(PRESETS))
def test_step_plans(checker, model, i8):
    c = PRESETS[model]
    ks = EXPECTED_KSPLIT.get((model, i8), "1 1 1 1 1" if not i8 else "-")
    args = [str(checker), str(c.hidden), str(c.intermediate), str(c.heads), str(c.kv_heads), str(c.head_dim),
            str(c.vocab), str(int(c.tied_embeddings)), str(int(i8))] + ks.split()
    r = subprocess.run(args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
