"""ctypes bindings of `libseedplane_cuda.so` (the C ABI declared in `include/seedplane_cuda.h`).

There is no fallback: if the library is missing or fails to load, importing the engine raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libseedplane_cuda.so"

SP_OK = 0
SP_ERR_INVALID = -1
SP_ERR_CUDA = -2
SP_ERR_CAPACITY = -3
SP_ERR_UNSUPPORTED = -4
SP_ERR_DEVICE = -5
SP_WEIGHTS_F16 = 0
SP_WEIGHTS_I8_B32 = 1

# Every symbol the header declares (the CPU tests check the library exports all of them).
EXPORTED = ("sp_last_error", "sp_version", "sp_engine_create", "sp_engine_destroy", "sp_engine_device_bytes",
            "sp_kv_create", "sp_kv_destroy", "sp_kv_length", "sp_kv_capacity", "sp_kv_set_length",
            "sp_forward", "sp_decode", "sp_decode_batch", "sp_prefill_batch", "sp_verify_tree", "sp_kv_commit", "sp_kv_copy", "sp_argmax", "sp_argmax_noalloc", "sp_mcol_gemm", "sp_topk",
            "sp_accept_stochastic", "sp_accept_greedy", "sp_sample_filter",
            "sp_device_status",
            "sp_trace_read")


class SpConfig(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("heads", C.c_int32), ("kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("intermediate", C.c_int32), ("vocab", C.c_int32),
                ("max_positions", C.c_int32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
                ("tied_embeddings", C.c_int32), ("weight_format", C.c_int32)]


class SpLayerWeights(C.Structure):
    _fields_ = [("qkv_w", C.c_void_p), ("qkv_s", C.c_void_p), ("qkv_b", C.c_void_p),
                ("o_w", C.c_void_p), ("o_s", C.c_void_p),
                ("gate_w", C.c_void_p), ("gate_s", C.c_void_p),
                ("up_w", C.c_void_p), ("up_s", C.c_void_p),
                ("down_w", C.c_void_p), ("down_s", C.c_void_p),
                ("in_norm", C.c_void_p), ("post_norm", C.c_void_p)]


class SpWeights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("lm_head", C.c_void_p), ("lm_head_s", C.c_void_p),
                ("final_norm", C.c_void_p), ("layers", C.POINTER(SpLayerWeights)), ("rope_host", C.c_void_p)]


_lib = None


def load(path: Path = LIB_PATH):
    """Load the engine library once; raises if it is absent (no CPU or library fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not Path(path).is_file():
        raise FileNotFoundError(f"{path} is missing: build it with `python -m seedplane_b200.build`")
    lib = C.CDLL(str(path))
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    pi32 = C.POINTER(C.c_int32)
    sig = {
        "sp_last_error": (C.c_char_p, []),
        "sp_version": (C.c_char_p, []),
        "sp_engine_create": (C.c_int, [C.POINTER(SpConfig), C.POINTER(SpWeights), C.c_int, C.POINTER(vp)]),
        "sp_engine_destroy": (None, [vp]),
        "sp_engine_device_bytes": (i64, [vp]),
        "sp_kv_create": (C.c_int, [vp, i32, C.POINTER(vp)]),
        "sp_kv_destroy": (None, [vp]),
        "sp_kv_length": (i32, [vp]),
        "sp_kv_capacity": (i32, [vp]),
        "sp_kv_set_length": (C.c_int, [vp, i32]),
        "sp_forward": (C.c_int, [vp, vp, vp, vp, i32, vp, i32, vp, vp]),
        "sp_decode": (C.c_int, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "sp_decode_batch": (C.c_int, [vp, C.POINTER(vp), i32, pi32, pi32, i32, vp, vp]),
        "sp_prefill_batch": (C.c_int, [vp, C.POINTER(vp), i32, vp, pi32, vp, vp]),
        "sp_verify_tree": (C.c_int, [vp, vp, pi32, pi32, i32, i32, vp, vp, vp]),
        "sp_kv_commit": (C.c_int, [vp, pi32, i32, vp]),
        "sp_kv_copy": (C.c_int, [vp, i32, vp, i32, i32, vp]),
        "sp_argmax": (C.c_int, [vp, vp, i32, i32, i64, vp, vp]),
        "sp_argmax_noalloc": (C.c_int, [C.c_int, vp, i32, i32, i64, vp, vp]),
        "sp_mcol_gemm": (C.c_int, [vp, i32, vp, vp, C.c_float, i32, i32, vp, i32, i32, i32, vp, i32, vp, vp, i32, vp]),
        "sp_topk": (C.c_int, [vp, vp, i32, i32, i64, i32, vp, vp, vp, vp]),
        "sp_accept_stochastic": (C.c_int, [vp, vp, vp, i64, i32, pi32, pi32, i32, C.c_double, C.c_uint64,
                                           C.c_uint64, pi32, vp]),
        "sp_accept_greedy": (C.c_int, [vp, vp, i32, pi32, pi32, i32, pi32, i32, pi32, vp]),
        "sp_sample_filter": (C.c_int, [vp, i32, C.c_double, i32, C.c_double, vp, vp]),
        "sp_device_status": (C.c_int, [vp, vp]),
        "sp_trace_read": (i64, [vp, C.POINTER(C.c_uint64), i64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class EngineError(RuntimeError):
    """A failed engine call (the code and the library's message)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (code {code})")
        self.code = code


def check(rc: int):
    if rc != SP_OK:
        msg = load().sp_last_error().decode("utf-8", "replace")
        if rc == SP_ERR_CAPACITY or rc == SP_ERR_INVALID:
            raise ValueError(msg)
        raise EngineError(rc, msg)
    return rc


def int_array(values):
    arr = (C.c_int32 * max(1, len(values)))(*[int(v) for v in values])
    return arr
