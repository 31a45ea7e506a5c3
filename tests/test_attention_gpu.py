"""Parity of the sm_100a attention kernel (through the C ABI) with the CPU
oracle and with the reference's own outputs (golden vectors).

Tolerance: max abs error <= 2e-2 and mean abs error
<= 2e-3 against the fp32 oracle, for bf16 inputs with fp32 accumulation.
"""

import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_close
import oracle
from cs348k_fast_attention_grammar_b200 import (FaError, attention, attention_bshd,
                                                attention_f32, attention_from_host,
                                                device_status)
from cs348k_fast_attention_grammar_b200 import kernel_module
from cs348k_fast_attention_grammar_b200.inputs import ATTN_CONFIGS, make_qkv

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _rand(shape, seed, amp=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * amp).to(torch.bfloat16)


def _run(q, k, v, causal):
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=DEV)
    attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal, out=out)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,S", [(1, 2, 128), (2, 3, 256), (1, 2, 384), (1, 1, 200),
                                   (1, 2, 1000), (1, 1, 1), (1, 1, 130), (2, 1, 512)])
def test_attention_matches_oracle(B, H, S, D, causal):
    q, k, v = (_rand((B, H, S, D), 10 + i) for i in range(3))
    out = _run(q, k, v, causal)
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                           causal=causal)
    assert_close(out, ref, what=f"B{B} H{H} S{S} D{D} causal={causal}")


@pytest.mark.parametrize("name", ["attn_program_N512_d64", "attn_program_N256_d128",
                                  "attn_program_N128_d64", "attn_best_it24_N512_d64"])
def test_attention_matches_reference_program(name):
    """Golden vectors from the reference's emitted cuTile programs (run through
    its numpy stand-in); inputs are bf16 values, layout KT [d, N]."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    out = kernel_module.fn(torch.from_numpy(z["KT"]).to(DEV), torch.from_numpy(z["Q"]).to(DEV),
                           torch.from_numpy(z["V"]).to(DEV))
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["O"], what=name)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N", [512, 200, 1000, 1])
@pytest.mark.parametrize("k_transposed", [True, False])
def test_attention_f32_matches_oracle(N, D, causal, k_transposed):
    """The fp32 2-D entry point (device-side bf16 staging, fp32 output):
    against the oracle on the bf16-rounded inputs (standard tolerance) and on
    the fp32 inputs themselves (looser bound covering the input rounding)."""
    g = torch.Generator().manual_seed(N * 7 + D + int(causal))
    q, k, v = (torch.randn((N, D), generator=g) for _ in range(3))
    kin = k.t().contiguous() if k_transposed else k
    out = attention_f32(q.to(DEV), kin.to(DEV), v.to(DEV), causal=causal,
                        k_transposed=k_transposed)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and tuple(out.shape) == (N, D)
    r = lambda t: t.to(torch.bfloat16).float().numpy()[None, None]  # noqa: E731
    ref = oracle.attention(r(q), r(k), r(v), causal=causal)[0, 0]
    assert_close(out.cpu().numpy(), ref, what=f"f32 N{N} D{D} causal={causal}")
    ref32 = oracle.attention(q.numpy()[None, None], k.numpy()[None, None], v.numpy()[None, None],
                             causal=causal)[0, 0]
    assert_close(out.cpu().numpy(), ref32, max_tol=5e-2, mean_tol=5e-3, what="f32 vs fp32 inputs")


def test_attention_f32_errors():
    q = torch.randn(512, 64, device=DEV)
    with pytest.raises(TypeError):
        attention_f32(q.half(), q.half(), q.half())
    with pytest.raises(ValueError):
        attention_f32(q, q[:256], q)
    with pytest.raises(FaError, match="head dimension"):
        x = torch.randn(512, 20, device=DEV)            # not a multiple of 8
        attention_f32(x, x, x)


def test_attention_matches_sota_module():
    z = np.load(os.path.join(GOLDEN, "sdpa_N512_d64.npz"))
    out = kernel_module.sota_fn(*(torch.from_numpy(z[n]).to(DEV) for n in ("K", "Q", "V")))
    assert_close(out.cpu().numpy(), z["O"], what="sdpa_N512_d64")


@pytest.mark.parametrize("name", ["sdpa_causal_S384_d128", "sdpa_causal_S200_d64"])
def test_attention_causal_matches_sdpa_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    q, k, v = (torch.from_numpy(z[n]).to(torch.bfloat16) for n in ("Q", "K", "V"))
    out = _run(q, k, v, causal=True)
    assert_close(out, z["O"], what=name)


def test_bshd_layout_is_bit_identical():
    B, S, H, D = 2, 384, 3, 128
    q, k, v = (_rand((B, S, H, D), 20 + i).to(DEV) for i in range(3))
    o1 = attention_bshd(q, k, v, causal=True)
    o2 = attention(q.permute(0, 2, 1, 3).contiguous(), k.permute(0, 2, 1, 3).contiguous(),
                   v.permute(0, 2, 1, 3).contiguous(), causal=True)
    torch.cuda.synchronize()
    assert torch.equal(o1.permute(0, 2, 1, 3), o2)


@pytest.mark.parametrize("chunks", [1, 2, 8])
def test_from_host_matches_device_call(chunks):
    """Chunked, stream-pipelined host path == one device call, bit for bit
    (3 pairs: chunk counts above the pair count are clamped)."""
    q, k, v = (_rand((1, 3, 384, 128), 30 + i).pin_memory() for i in range(3))
    ws = {}
    for _ in range(2):                       # reuses the workspace on the 2nd call
        o_host = attention_from_host(q, k, v, causal=True, device=DEV, workspace=ws,
                                     chunks=chunks)
        torch.cuda.synchronize()
        o_dev = attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=True)
        assert torch.equal(o_host, o_dev.cpu())


def test_repeated_calls_are_deterministic():
    q, k, v = (_rand((2, 4, 1024, 128), 40 + i).to(DEV) for i in range(3))
    a = attention(q, k, v, causal=True)
    b = attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert device_status() == 0


def test_error_codes():
    q = _rand((1, 1, 128, 136), 1).to(DEV)              # above the largest head dim
    with pytest.raises(FaError, match="head dimension"):
        attention(q, q, q)
    ok = _rand((1, 1, 128, 64), 2).to(DEV)
    flat = torch.zeros(128 * 65 + 64, dtype=torch.bfloat16, device=DEV)
    odd = flat.as_strided((1, 1, 128, 64), (128 * 65, 128 * 65, 65, 1))   # row stride 130 B
    with pytest.raises(FaError, match="aligned"):
        attention(odd, ok, ok)
    with pytest.raises(FaError, match="innermost stride"):
        attention(ok.transpose(2, 3).contiguous().transpose(2, 3), ok, ok)
    with pytest.raises(ValueError):
        attention(q.cpu(), q.cpu(), q.cpu())
    with pytest.raises(TypeError):
        attention(ok.to(torch.int16), ok.to(torch.int16), ok.to(torch.int16))
    with pytest.raises(TypeError):
        attention(ok, ok.half(), ok)                     # mixed dtypes


# ---------------------------------------------------------------------------
# Full BASELINE sizes: a seeded subset of pairs against a torch fp32
# reference on the GPU, plus size-independent properties.
# ---------------------------------------------------------------------------
def _torch_ref_pair(q, k, v, causal, row_chunk=2048):
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


@pytest.mark.parametrize("cfg_name", ["cfg1", "cfg2"])
def test_full_size_subset(cfg_name):
    cfg = ATTN_CONFIGS[cfg_name]
    npairs = cfg["B"] * cfg["H"]
    q, k, v = make_qkv(cfg, range(npairs), DEV)
    q = q.view(cfg["B"], cfg["H"], cfg["S"], cfg["D"])
    k = k.view_as(q)
    v = v.view_as(q)
    o = attention(q, k, v, causal=cfg["causal"])
    rng = np.random.default_rng(123)
    for p in rng.choice(npairs, size=4, replace=False):
        b, h = divmod(int(p), cfg["H"])
        ref = _torch_ref_pair(q[b, h], k[b, h], v[b, h], cfg["causal"])
        d = (o[b, h].float() - ref).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, (cfg_name, p, d.max().item())
    assert torch.isfinite(o.float()).all()


def test_property_constant_v_gives_constant_output():
    """Rows of P sum to one: V = c everywhere gives O = c (all S, causal)."""
    B, H, S, D = 1, 2, 3000, 128
    q, k = _rand((B, H, S, D), 50).to(DEV), _rand((B, H, S, D), 51).to(DEV)
    v = torch.full((B, H, S, D), 0.75, dtype=torch.bfloat16, device=DEV)
    for causal in (False, True):
        o = attention(q, k, v, causal=causal).float()
        assert (o - 0.75).abs().max().item() < 4e-3


def test_property_causal_first_row_is_v0():
    B, H, S, D = 1, 2, 2048, 64
    q, k, v = (_rand((B, H, S, D), 60 + i).to(DEV) for i in range(3))
    o = attention(q, k, v, causal=True)
    assert (o[:, :, 0].float() - v[:, :, 0].float()).abs().max().item() < 1e-2


def test_property_key_permutation_invariance():
    """Non-causal attention is invariant under a joint permutation of K/V rows."""
    B, H, S, D = 1, 2, 1024, 128
    q, k, v = (_rand((B, H, S, D), 70 + i).to(DEV) for i in range(3))
    perm = torch.randperm(S, generator=torch.Generator().manual_seed(0)).to(DEV)
    o1 = attention(q, k, v).float()
    o2 = attention(q, k[:, :, perm].contiguous(), v[:, :, perm].contiguous()).float()
    assert (o1 - o2).abs().max().item() < 2e-2


@pytest.mark.parametrize("shape", [(0, 2, 128, 64), (1, 0, 128, 128), (2, 3, 0, 64)])
def test_empty_inputs_return_empty_output(shape):
    """Like torch SDPA, an empty batch, head or sequence axis gives an empty
    result (no launch, no error)."""
    q = torch.empty(shape, dtype=torch.bfloat16, device=DEV)
    o = attention(q, q, q, causal=True)
    assert tuple(o.shape) == shape


@pytest.mark.parametrize("D,causal", [(64, True), (128, False)])
def test_long_sequence_one_pair(D, causal):
    """S = 65536 (512 key blocks, 256 units per head): rows spread over the
    sequence against a torch fp32 reference, plus finiteness everywhere."""
    S = 65536
    q, k, v = (_rand((1, 1, S, D), 80 + i, amp=0.5).to(DEV) for i in range(3))
    o = attention(q, k, v, causal=causal)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    qf, kf, vf = q[0, 0].float(), k[0, 0].float(), v[0, 0].float()
    rows = torch.tensor([0, 1, 127, 128, 4095, 30000, 65535], device=DEV)
    s = (qf[rows] @ kf.t()) / math.sqrt(D)
    if causal:
        s = s.masked_fill(torch.arange(S, device=DEV)[None, :] > rows[:, None], float("-inf"))
    ref = torch.softmax(s, dim=-1) @ vf
    d = (o[0, 0, rows].float() - ref).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, d.max().item()


def _random_cases(n=40, seed=2026):
    rng = np.random.default_rng(seed)
    cases = []
    for _ in range(n):
        D = int(rng.choice([64, 128]))
        S = int(rng.choice([int(rng.integers(1, 1100)), int(rng.choice([64, 128, 256, 512, 640]))]))
        B = int(rng.integers(1, 3))
        H = int(rng.integers(1, 4))
        causal = bool(rng.integers(0, 2))
        layout = str(rng.choice(["bhsd", "bshd", "padded"]))
        cases.append((B, H, S, D, causal, layout))
    return cases


@pytest.mark.parametrize("B,H,S,D,causal,layout", _random_cases())
def test_attention_random_shapes_and_layouts(B, H, S, D, causal, layout):
    """Seeded random shapes (ragged S, both head dims, causal or not) and
    memory layouts: contiguous [B,H,S,D], (B,S,H,D) viewed as [B,H,S,D], and
    rows padded to a larger sequence stride."""
    g = torch.Generator().manual_seed(B * 1000003 + H * 1009 + S * 7 + D + int(causal))
    if layout == "bhsd":
        mk = lambda: torch.randn((B, H, S, D), generator=g).to(torch.bfloat16)  # noqa: E731
    elif layout == "bshd":
        mk = lambda: torch.randn((B, S, H, D), generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)  # noqa
    else:
        mk = lambda: torch.randn((B, H, S + 24, D), generator=g).to(torch.bfloat16)[:, :, :S]  # noqa
    q, k, v = mk(), mk(), mk()
    out = attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    torch.cuda.synchronize()
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal)
    assert_close(out.float().cpu().numpy(), ref, what=f"{layout} B{B} H{H} S{S} D{D} c={causal}")


def _units(B, H, S, D):
    rows = 512 if D == 64 else 256      # query rows per work unit
    return B * H * ((S + rows - 1) // rows)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_persistent_launch_matches_oracle(D, causal):
    """More work units than SMs: the kernel runs persistent, one CTA per SM
    taking units from a global counter.  Every head is checked."""
    B, H, S = 1, 160, 384
    assert _units(B, H, S, D) > torch.cuda.get_device_properties(0).multi_processor_count
    q, k, v = (_rand((B, H, S, D), 70 + i) for i in range(3))
    out = _run(q, k, v, causal)
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                           causal=causal)
    assert_close(out, ref, what=f"persistent H{H} S{S} D{D} causal={causal}")


def test_persistent_counter_pairs_wrap_and_reset():
    """1100 persistent launches use every one of the 1024 counter pairs and
    wrap around, so each pair must be left at zero by the launch before."""
    q, k, v = (_rand((1, 160, 256, 128), 80 + i).to(DEV) for i in range(3))
    first = attention(q, k, v, causal=True)
    out = torch.empty_like(first)
    for _ in range(1100):
        attention(q, k, v, causal=True, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert device_status() == 0


def test_persistent_launches_on_two_streams():
    """Persistent launches in flight on two streams at once take different
    counter pairs; each stream's results equal its single-launch output."""
    ins = [[_rand((1, 160, 512, 128), 90 + 3 * s + i).to(DEV) for i in range(3)]
           for s in range(2)]
    want = [attention(*x, causal=bool(s)) for s, x in enumerate(ins)]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty_like(w) for w in want]
    bad = [0, 0]
    for _ in range(40):
        for s in range(2):
            with torch.cuda.stream(streams[s]):
                attention(*ins[s], causal=bool(s), out=outs[s])
        for s in range(2):
            streams[s].synchronize()
            bad[s] += int(not torch.equal(outs[s], want[s]))
    assert bad == [0, 0]
    assert device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_score_jump_in_later_block(dtype, D, causal):
    """A key in a later key block scores far above everything before it for
    some rows (more than 64 in log2 units, beyond the range the softmax keeps
    against its running reference maximum), so those rows take the exact
    path: block maximum, O rescaled, probabilities redone.  Other rows of the
    same warps stay on the fast path.  Checked against the fp64 oracle."""
    S = 512
    g = torch.Generator().manual_seed(400 + D + int(causal))
    q, k, v = (torch.randn((1, 2, S, D), generator=g) for _ in range(3))
    q[:, :, 320:400] = 3.0          # these rows ...
    k[:, :, 300] = 3.0              # ... meet this key in key block 2 (or 4)
    k[:, 1, 450] = 2.0              # a smaller jump in head 1
    q, k, v = (t.to(dtype) for t in (q, k, v))
    out = attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    torch.cuda.synchronize()
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal)
    assert_close(out.float().cpu().numpy(), ref, what=f"{dtype} D{D} causal={causal}")
    assert device_status() == 0


@pytest.mark.parametrize("S", [1024, 1000])
def test_split_last_wave_matches_oracle(S):
    """Non-causal D = 64 with a last partial wave of r <= SMs / 2 equal units:
    those units run as half units (two per unit).  S = 1024 fills every unit,
    S = 1000 leaves each head's last unit 488 of 512 rows.  Every head is
    checked against the oracle."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    H = (sms + 12) // 2                  # 2 units per head: units = sms + 12 (or 11)
    q, k, v = (_rand((1, H, S, 64), 90 + i) for i in range(3))
    out = _run(q, k, v, False)
    ref = oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False)
    assert_close(out, ref, what=f"split tail S={S} H={H}")
    assert device_status() == 0
