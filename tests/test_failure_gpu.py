"""Failure detection on the GPU without a fault: a kernel wait that nothing
completes runs out after its short limit, the kernel records FA_ERR_TIMEOUT in
the device status word and returns, the host reads the status, and the
context keeps working (the next attention call is correct)."""

import numpy as np
import pytest
import torch

import oracle
from cs348k_fast_attention_grammar_b200 import _lib, attention, device_status

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
FA_ERR_TIMEOUT = 11


def test_bounded_wait_times_out_and_context_survives():
    lib = _lib.load()
    assert device_status() == 0                       # clean before
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.fa_selftest_wait_timeout(2000, stream)   # 2 ms limit
    assert rc == 0, _lib.strerror(rc)
    assert device_status() == FA_ERR_TIMEOUT          # reported ...
    assert device_status() == 0                       # ... and cleared by the read
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 2, 256, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    o = attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=True)
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True)
    assert np.abs(o.float().cpu().numpy() - ref).max() <= 2e-2
    assert device_status() == 0


def test_selftest_rejects_bad_limits():
    lib = _lib.load()
    assert lib.fa_selftest_wait_timeout(0, None) == 10      # FA_ERR_ARG
    assert lib.fa_selftest_wait_timeout(2_000_000, None) == 10
