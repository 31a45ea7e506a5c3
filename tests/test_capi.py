"""The C-ABI library: it loads on a machine without a GPU, exports every
symbol include/fa_b200.h declares, and its host-side argument checks return
the documented status codes before any device work.  No compute calls."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from cs348k_fast_attention_grammar_b200 import _lib

HEADER = os.path.join(ROOT, "include", "fa_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z0-9_]+)\s*\(", text)))


def _declared_status_codes():
    text = open(HEADER).read()
    return {m[0]: int(m[1]) for m in re.findall(r"\b(FA_(?:OK|ERR_[A-Z_]+))\s*=\s*(\d+)", text)}


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared_functions()
    assert {"fa_attn_fwd", "fa_mlp_fwd", "fa_gemm_act", "fa_strerror"} <= set(names)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in fa_b200.h but not exported"


def test_python_binding_covers_header():
    bound = set(_lib.SIGNATURES)
    declared = set(_declared_functions())
    assert bound == declared


def test_strerror_for_every_status_code():
    codes = _declared_status_codes()
    assert codes["FA_OK"] == 0 and len(codes) >= 13
    texts = {c: _lib.strerror(v) for c, v in codes.items()}
    assert texts["FA_OK"] == "success"
    assert len(set(texts.values())) == len(texts)          # all distinct
    assert _lib.strerror(999) == "unknown fa_status"


def test_version():
    assert _lib.load().fa_version() >= 100


def test_argument_checks_without_device():
    """Checks that run before any CUDA call return their codes on a CPU box."""
    lib = _lib.load()
    st = (ctypes.c_int64 * 16)(*([8192, 1024, 64, 1] * 4))
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(258)
    codes = _declared_status_codes()
    assert lib.fa_attn_fwd(None, p, p, p, 1, 1, 16, 64, st, 0, 0.125, None) == codes["FA_ERR_NULL"]
    assert lib.fa_attn_fwd(p, p, p, p, 0, 1, 16, 64, st, 0, 0.125, None) == codes["FA_ERR_SHAPE"]
    for bad_d in (100, 136, 0, 4):          # not a multiple of 8, or outside 8..128
        assert lib.fa_attn_fwd(p, p, p, p, 1, 1, 16, bad_d, st, 0, 0.125, None) == \
            codes["FA_ERR_HEAD_DIM"]
        assert lib.fa_attn_fwd_f16(p, p, p, p, 1, 1, 16, bad_d, st, 0, 0.125, None) == \
            codes["FA_ERR_HEAD_DIM"]
    assert lib.fa_attn_fwd_f16(None, p, p, p, 1, 1, 16, 64, st, 0, 0.125, None) == \
        codes["FA_ERR_NULL"]
    b32 = lib.fa_attn_fwd_f32_batched
    assert b32(p, p, p, p, None, 1, 4, 256, 64, 0, 0, 0.125, 0, None) == codes["FA_ERR_NULL"]
    assert b32(p, p, p, p, p, 1, 0, 256, 64, 0, 0, 0.125, 0, None) == codes["FA_ERR_SHAPE"]
    assert b32(p, p, p, p, p, 1, 4, 256, 64, 2, 0, 0.125, 0, None) == codes["FA_ERR_SHAPE"]
    assert b32(p, p, p, p, p, 1, 4, 256, 76, 0, 0, 0.125, 0, None) == codes["FA_ERR_HEAD_DIM"]
    assert b32(p, p, p, p, p, 1, 4, 256, 72, 0, 0, 0.125, 1, None) == codes["FA_ERR_HEAD_DIM"]
    assert b32(p, p, p, p, p, 1, 4, 256, 64, 0, 0, 0.125, 2, None) == codes["FA_ERR_ARG"]
    assert b32(p, p, p, odd, p, 1, 4, 256, 64, 0, 0, 0.125, 0, None) == codes["FA_ERR_ALIGN"]
    bad = (ctypes.c_int64 * 16)(*([8192, 1024, 65, 1] * 4))
    assert lib.fa_attn_fwd(p, p, p, p, 1, 1, 16, 64, bad, 0, 0.125, None) == codes["FA_ERR_ALIGN"]
    bad = (ctypes.c_int64 * 16)(*([8192, 1024, 64, 2] * 4))
    assert lib.fa_attn_fwd(p, p, p, p, 1, 1, 16, 64, bad, 0, 0.125, None) == \
        codes["FA_ERR_STRIDE"]
    assert lib.fa_attn_fwd(odd, p, p, p, 1, 1, 16, 64, st, 0, 0.125, None) == \
        codes["FA_ERR_ALIGN"]
    f32 = lib.fa_attn_fwd_f32
    assert f32(p, p, p, p, None, 512, 64, 1, 0, 0.125, None) == codes["FA_ERR_NULL"]
    assert f32(p, p, p, p, p, 0, 64, 1, 0, 0.125, None) == codes["FA_ERR_SHAPE"]
    assert f32(p, p, p, p, p, 512, 64, 2, 0, 0.125, None) == codes["FA_ERR_SHAPE"]
    assert f32(p, p, p, p, p, 512, 20, 1, 0, 0.125, None) == codes["FA_ERR_HEAD_DIM"]
    assert f32(p, p, p, p, odd, 512, 64, 1, 0, 0.125, None) == codes["FA_ERR_ALIGN"]
    assert lib.fa_gemm_act(p, p, p, 128, 100, 64, 64, 100, 100, 0, None) == codes["FA_ERR_SHAPE"]
    assert lib.fa_gemm_act(p, p, p, 128, 128, 64, 64, 128, 128, 7, None) == codes["FA_ERR_ARG"]
    assert lib.fa_gemm_act(p, p, p, 128, 128, 64, 60, 128, 128, 0, None) == \
        codes["FA_ERR_STRIDE"]
    assert lib.fa_gemm_act_f16(p, p, p, 128, 100, 64, 64, 100, 100, 0, None) == \
        codes["FA_ERR_SHAPE"]
    assert lib.fa_mlp_fwd_f16(p, p, p, None, p, 128, 64, 256, 2, None) == codes["FA_ERR_NULL"]
    assert lib.fa_selftest_wait_timeout(0, None) == codes["FA_ERR_ARG"]
    fn = lib.fa_mlp_fwd_noalloc
    assert fn(p, p, p, p, 4096, 64, 4096, 2, None) == codes["FA_ERR_SCRATCH"]
    assert fn(p, p, p, p, 2049, 64, 4096, 2, None) == codes["FA_ERR_SCRATCH"]
    # argument checks precede every CUDA call, so they hold without a device
    assert fn(None, p, p, p, 128, 64, 256, 2, None) == codes["FA_ERR_NULL"]
    assert fn(p, p, p, None, 128, 64, 256, 2, None) == codes["FA_ERR_NULL"]
    assert fn(p, p, p, p, 128, 64, 100, 2, None) == codes["FA_ERR_SHAPE"]
    assert fn(p, p, p, p, 128, 60, 256, 2, None) == codes["FA_ERR_SHAPE"]
    assert fn(p, p, p, p, 0, 64, 256, 2, None) == codes["FA_ERR_SHAPE"]
    assert fn(p, p, p, p, 128, 64, 256, 9, None) == codes["FA_ERR_ARG"]
    assert fn(odd, p, p, p, 128, 64, 256, 2, None) == codes["FA_ERR_ALIGN"]


def test_no_cpu_fallback_in_package():
    """The product package never imports the oracle."""
    pkg = os.path.join(ROOT, "cs348k_fast_attention_grammar_b200")
    for fn in os.listdir(pkg):
        if fn.endswith(".py"):
            src = open(os.path.join(pkg, fn)).read()
            assert "import oracle" not in src and "from oracle" not in src, fn
