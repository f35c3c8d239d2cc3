"""The C ABI library on the CPU: it builds, loads, exports every symbol the header declares, and
rejects bad arguments with an error code and message (no GPU is touched by these calls)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from seedplane_b200 import _native as N
from seedplane_b200.build import LIB, build

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    build()  # no-op when up to date
    return N.load()


def declared_functions():
    text = (ROOT / "include" / "seedplane_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(sp_[a-z_0-9]+)\s*\(", text))


def test_header_and_binding_list_agree():
    assert declared_functions() == set(N.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    raw = C.CDLL(str(LIB))
    for name in declared_functions():
        assert hasattr(raw, name), name
    assert lib.sp_version().decode().startswith("seedplane-b200")


def test_null_arguments_are_rejected_with_messages(lib):
    h = C.c_void_p()
    rc = lib.sp_engine_create(None, None, 0, C.byref(h))
    assert rc == N.SP_ERR_INVALID
    assert "null" in lib.sp_last_error().decode()
    assert lib.sp_kv_length(None) == -1
    assert lib.sp_kv_capacity(None) == -1
    assert lib.sp_kv_set_length(None, 0) == N.SP_ERR_INVALID
    assert lib.sp_kv_commit(None, None, 0, None) == N.SP_ERR_INVALID
    assert lib.sp_kv_copy(None, 0, None, 0, 1, None) == N.SP_ERR_INVALID
    assert lib.sp_decode_batch(None, None, 1, None, None, 1, None, None) == N.SP_ERR_INVALID
    assert lib.sp_prefill_batch(None, None, 1, None, None, None, None) == N.SP_ERR_INVALID
    assert lib.sp_device_status(None, None) == N.SP_ERR_INVALID
    assert lib.sp_argmax(None, None, 1, 1, 1, None, None) == N.SP_ERR_INVALID
    assert lib.sp_argmax_noalloc(0, None, 1, 1, 1, None, None) == N.SP_ERR_INVALID
    # more rows than the fixed scratch holds: rejected before any CUDA call
    assert lib.sp_argmax_noalloc(0, C.c_void_p(256), 129, 8, 8, C.c_void_p(256), None) == N.SP_ERR_CAPACITY
    with pytest.raises(ValueError):
        N.check(N.SP_ERR_INVALID)


def test_bad_config_is_rejected_before_touching_a_device(lib):
    cfg = N.SpConfig(layers=2, hidden=100, heads=3, kv_heads=1, head_dim=33, intermediate=64, vocab=10,
                     max_positions=16, rope_theta=1e6, rms_norm_eps=1e-6, tied_embeddings=1, weight_format=0)
    w = N.SpWeights()
    h = C.c_void_p()
    assert lib.sp_engine_create(C.byref(cfg), C.byref(w), 0, C.byref(h)) == N.SP_ERR_INVALID
    assert "head" in lib.sp_last_error().decode()
    cfg = N.SpConfig(layers=2, hidden=96, heads=3, kv_heads=1, head_dim=32, intermediate=64, vocab=10,
                     max_positions=16, rope_theta=1e6, rms_norm_eps=1e-6, tied_embeddings=1, weight_format=0)
    assert lib.sp_engine_create(C.byref(cfg), C.byref(w), 0, C.byref(h)) == N.SP_ERR_UNSUPPORTED
    assert "head_dim" in lib.sp_last_error().decode()
