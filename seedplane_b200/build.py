"""Build the engine library `seedplane_b200/libseedplane_cuda.so` in tree with nvcc for sm_100a.

    python -m seedplane_b200.build [--force] [--verbose]

The library is a plain shared object exporting the C ABI of `include/seedplane_cuda.h`; the
CUDA runtime is linked statically, so it loads next to PyTorch's own runtime without conflict.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libseedplane_cuda.so"
SOURCES = ["kernels.cu", "gemv_tc.cu", "attention.cu", "argmax.cu", "step.cu", "prefill.cu", "mcol.cu", "sample.cu", "engine.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _inputs():
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date(lib: Path = LIB) -> bool:
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> Path:
    if not force and up_to_date():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    common = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr", *extra_flags]
    if verbose:
        common += ["-Xptxas", "-v"]
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/shared-memory usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
