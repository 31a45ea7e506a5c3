"""The BASELINE configurations on their own seeded inputs, end to end on the
GPU, against the fp32 oracle / reference -- the same checks the reference's
search makes on its seeded problem (run_attention_search.py:169-181) -- plus
the softmax's exponential routines run on the device.

* cfg0: fp32 B1 H4 S256 D64, seed 0 (the CPU-runnable configuration), through
  the batched bf16 entry point and, pair by pair, through the fp32 entry
  point, against the oracle.
* cfg4: causal bf16 B64 H32 S16384 D128, seed 4: all 2048 (batch, head) pairs
  in one launch on one GPU (the 8-GPU run shards exactly these pairs, and a
  pair's output does not depend on the sharding), checked on the 32 seeded
  pairs bench.py verifies, against a chunked fp32 reference.
"""

import math

import numpy as np
import pytest
import torch

from conftest import assert_close
import oracle
from cs348k_fast_attention_grammar_b200 import _lib, attention, attention_f32, device_status
from cs348k_fast_attention_grammar_b200.inputs import ATTN_CONFIGS, make_qkv
from cs348k_fast_attention_grammar_b200.parallel import verify_pairs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _chunked_ref(q, k, v, causal, row_chunk=2048):
    qf, kf, vf = q.float(), k.float(), v.float()
    S, D = qf.shape
    out = torch.empty_like(qf)
    for r0 in range(0, S, row_chunk):
        s = (qf[r0:r0 + row_chunk] @ kf.t()) / math.sqrt(D)
        if causal:
            rows = torch.arange(r0, min(S, r0 + row_chunk), device=q.device)[:, None]
            s = s.masked_fill(torch.arange(S, device=q.device)[None, :] > rows, float("-inf"))
        out[r0:r0 + row_chunk] = torch.softmax(s, dim=-1) @ vf
    return out


def test_cfg0_seeded_inputs():
    cfg = ATTN_CONFIGS["cfg0"]
    B, H, S, D = cfg["B"], cfg["H"], cfg["S"], cfg["D"]
    q, k, v = (t.view(B, H, S, D) for t in make_qkv(cfg, range(B * H), "cpu", torch.float32))
    qn, kn, vn = (t.numpy() for t in (q, k, v))
    ref32 = oracle.attention(qn, kn, vn, causal=cfg["causal"])
    rb = lambda t: t.to(torch.bfloat16).float().numpy()  # noqa: E731
    ref_b = oracle.attention(rb(q), rb(k), rb(v), causal=cfg["causal"])
    # batched bf16 entry point on the bf16-cast inputs
    o = attention(*(t.to(torch.bfloat16).to(DEV) for t in (q, k, v)), causal=cfg["causal"])
    torch.cuda.synchronize()
    assert_close(o.float().cpu().numpy(), ref_b, what="cfg0 bf16 entry vs oracle")
    # the fp32 tensors as given: one batched fp32 call (device-side staging)
    o32 = attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=cfg["causal"])
    torch.cuda.synchronize()
    assert o32.dtype == torch.float32 and tuple(o32.shape) == (B, H, S, D)
    assert_close(o32.cpu().numpy(), ref_b, what="cfg0 batched fp32 entry vs oracle")
    assert_close(o32.cpu().numpy(), ref32, max_tol=5e-2, mean_tol=5e-3,
                 what="cfg0 batched fp32 entry vs fp32 inputs")
    # fp32 entry point, one (batch, head) pair per call, fp32 output
    for h in range(H):
        of = attention_f32(q[0, h].to(DEV), k[0, h].to(DEV), v[0, h].to(DEV),
                           causal=cfg["causal"])
        torch.cuda.synchronize()
        assert of.dtype == torch.float32
        assert_close(of.cpu().numpy(), ref_b[0, h], what=f"cfg0 fp32 entry head {h}")
        assert_close(of.cpu().numpy(), ref32[0, h], max_tol=5e-2, mean_tol=5e-3,
                     what=f"cfg0 fp32 entry head {h} vs fp32 inputs")
        assert torch.equal(of, o32[0, h])     # same staging, same kernel, per pair


def test_cfg4_all_pairs_one_launch_seeded_subset():
    cfg = ATTN_CONFIGS["cfg4"]
    n = cfg["B"] * cfg["H"]
    q, k, v = make_qkv(cfg, range(n), DEV)            # [1, 2048, 16384, 128] each
    o = attention(q, k, v, causal=cfg["causal"])
    torch.cuda.synchronize()
    for p in verify_pairs(n, 32):
        ref = _chunked_ref(q[0, p], k[0, p], v[0, p], cfg["causal"])
        d = (o[0, p].float() - ref).abs()
        mx, mean = d.max().item(), d.mean().item()
        assert mx <= 2e-2 and mean <= 2e-3, (p, mx, mean)
    rows = torch.arange(0, o.shape[1], 97, device=DEV)
    assert torch.isfinite(o[0, rows].float()).all()
    assert device_status() == 0


def test_device_exp2_routines():
    """The FMA-pipe exp2 (scalar and paired) and ex2.approx as the attention
    kernels run them, over the softmax's range [-125, 8]: relative error
    against exp2 in fp64 within the polynomial's bound (1.2e-4), the paired
    routine equal to the scalar one bit for bit, and values below -125
    clamped to a tiny positive number."""
    lib = _lib.load()
    x = torch.cat([torch.linspace(-125.0, 8.0, 1 << 20), torch.tensor([-1e30, -200.0])])
    n = x.numel()
    xd = x.to(DEV)
    out = torch.empty(3 * n, device=DEV)
    rc = lib.fa_selftest_exp2(xd.data_ptr(), out.data_ptr(), n,
                              torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    o = out.cpu().numpy().reshape(3, n)
    xs = x.numpy()
    ref = np.exp2(xs[:-2].astype(np.float64))
    fma, fma2, mufu = o[0], o[1], o[2]
    assert np.max(np.abs(fma[:-2] / ref - 1.0)) < 1.2e-4
    np.testing.assert_array_equal(fma.view(np.int32), fma2.view(np.int32))
    assert np.max(np.abs(mufu[:-2] / ref - 1.0)) < 1e-6
    assert np.all(fma[-2:] > 0) and np.all(fma[-2:] < 1e-37)
