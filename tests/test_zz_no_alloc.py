"""fa_mlp_fwd_noalloc: the MLP block for callers that cannot allocate device
memory (a plugin inside a host that owns every memory pool, code that must not
allocate while a graph is built or while another component holds the memory
budget).  It keeps the hidden activation in a fixed 16 MiB array inside the
library instead of a caller buffer.

Called through the C ABI and compared with the allocating entry point
fa_mlp_fwd (caller-provided hidden buffer) on two calls in a row with
different inputs, so a stale hidden array from the previous call would show.
This file is named to be collected last.
"""

import numpy as np
import pytest
import torch

from conftest import assert_close
from cs348k_fast_attention_grammar_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
FA_ERR_SCRATCH = 13
MAX_HIDDEN_ELEMS = 8 * 1024 * 1024


def _noalloc_fn():
    lib = _lib.load()
    return lib, lib.fa_mlp_fwd_noalloc


def _inputs(M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (torch.randn(K, N, generator=g) / K ** 0.5).to(torch.bfloat16).to(DEV)
    w2 = (torch.randn(N, K, generator=g) / N ** 0.5).to(torch.bfloat16).to(DEV)
    return x, w1, w2


def test_noalloc_matches_allocating_mlp_twice():
    lib, fn = _noalloc_fn()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    calls = [(512, 256, 2048, "gelu_tanh", 11), (384, 192, 4096, "relu", 12)]
    for M, K, N, act, seed in calls:
        x, w1, w2 = _inputs(M, K, N, seed)
        a = _lib.ACTIVATIONS[act]
        hidden = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        y_ref = torch.empty(M, K, dtype=torch.bfloat16, device=DEV)
        rc = lib.fa_mlp_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), hidden.data_ptr(),
                            y_ref.data_ptr(), M, K, N, a, stream)
        assert rc == 0, _lib.strerror(rc)
        y = torch.full((M, K), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = fn(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), M, K, N, a, stream)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert_close(y.float().cpu().numpy(), y_ref.float().cpu().numpy(),
                     what=f"noalloc vs fa_mlp_fwd M{M} K{K} N{N} {act}")


def test_noalloc_at_its_limit_matches_fa_mlp_fwd_and_oracle():
    """The largest problem the fixed array takes (M * N exactly 8,388,608),
    large enough for the two-SM GEMM tiles, against the allocating entry point
    and, on a seeded subset of rows, against the CPU oracle."""
    import oracle
    lib, fn = _noalloc_fn()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    M, K, N = 2048, 256, 4096
    assert M * N == MAX_HIDDEN_ELEMS
    x, w1, w2 = _inputs(M, K, N, 21)
    a = _lib.FA_ACT_GELU_TANH
    hidden = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    y_ref = torch.empty(M, K, dtype=torch.bfloat16, device=DEV)
    assert lib.fa_mlp_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), hidden.data_ptr(),
                          y_ref.data_ptr(), M, K, N, a, stream) == 0
    y = torch.full((M, K), float("nan"), dtype=torch.bfloat16, device=DEV)
    rc = fn(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), M, K, N, a, stream)
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    yf = y.float().cpu().numpy()
    assert_close(yf, y_ref.float().cpu().numpy(), what="noalloc at the limit vs fa_mlp_fwd")
    rows = np.random.default_rng(5).choice(M, 64, replace=False)
    ref = oracle.mlp(x.float().cpu().numpy()[rows], w1.float().cpu().numpy(),
                     w2.float().cpu().numpy(), act="gelu_tanh", round_hidden_bf16=True)
    assert_close(yf[rows], ref, what="noalloc at the limit vs oracle")


def test_noalloc_rejects_hidden_larger_than_its_array():
    lib, fn = _noalloc_fn()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    for M, K, N in ((4096, 64, 4096), (2049, 64, 4096)):   # 2x, and one row over
        assert M * N > MAX_HIDDEN_ELEMS
        x = torch.empty(M, K, dtype=torch.bfloat16, device=DEV)
        w1 = torch.empty(K, N, dtype=torch.bfloat16, device=DEV)
        w2 = torch.empty(N, K, dtype=torch.bfloat16, device=DEV)
        y = torch.empty(M, K, dtype=torch.bfloat16, device=DEV)
        rc = fn(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), M, K, N,
                _lib.FA_ACT_GELU_TANH, stream)
        assert rc == FA_ERR_SCRATCH
        assert "fixed hidden buffer" in _lib.strerror(rc)
