"""ctypes binding of libfa_b200.so (the C ABI declared in include/fa_b200.h).

There is no fallback: if the library is missing or fails to load, every
operator raises.  ``load()`` builds the library in-tree first when its sources
are newer (the same build ``__graft_entry__.build()`` runs).
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

FA_OK = 0
FA_F32_BF16 = 0
FA_F32_SPLIT = 1
FA_ACT_NONE = 0
FA_ACT_RELU = 1
FA_ACT_GELU_TANH = 2
ACTIVATIONS = {"none": FA_ACT_NONE, "relu": FA_ACT_RELU, "gelu_tanh": FA_ACT_GELU_TANH}

# Every symbol include/fa_b200.h declares, with its ctypes signature.
_c_int, _c_float, _vp, _i64 = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int64
SIGNATURES = {
    "fa_strerror": (ctypes.c_char_p, [_c_int]),
    "fa_version": (_c_int, []),
    "fa_attn_fwd": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                             ctypes.POINTER(_i64), _c_int, _c_float, _vp]),
    "fa_attn_fwd_f16": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                 ctypes.POINTER(_i64), _c_int, _c_float, _vp]),
    "fa_attn_fwd_f32": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                 _c_float, _vp]),
    "fa_attn_fwd_f32_batched": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                         _c_int, _c_int, _c_int, _c_float, _c_int, _vp]),
    "fa_gemm_act": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _i64, _i64, _i64,
                             _c_int, _vp]),
    "fa_gemm_act_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _i64, _i64, _i64,
                                 _c_int, _vp]),
    "fa_mlp_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "fa_mlp_fwd_f16": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "fa_mlp_ln_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                               _c_float, _vp]),
    "fa_layernorm_rows": (_c_int, [_vp, _vp, _c_int, _c_int, _i64, _i64, _c_float, _vp]),
    "fa_mlp_fwd_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "fa_device_status": (_c_int, []),
    "fa_selftest_wait_timeout": (_c_int, [_c_int, _vp]),
    "fa_selftest_exp2": (_c_int, [_vp, _vp, _c_int, _vp]),
}

_lock = threading.Lock()
_lib = None


class FaError(RuntimeError):
    """A nonzero fa_status returned through the C ABI."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {strerror(code)} (fa_status {code})")


def load(build_if_stale: bool = True) -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_stale and (_build.is_stale()):
            _build.build()
        if not os.path.exists(_build.LIB_PATH):
            raise RuntimeError(f"{_build.LIB_PATH} is missing; run "
                               "python -m cs348k_fast_attention_grammar_b200.build")
        lib = ctypes.CDLL(_build.LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def strerror(code: int) -> str:
    return load().fa_strerror(int(code)).decode()


def check(code: int, where: str) -> None:
    if code != FA_OK:
        raise FaError(code, where)


def lib_path() -> str:
    return _build.LIB_PATH
