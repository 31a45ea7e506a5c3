"""The B200 backend for the reference's kernel grammar (``grammar_backend``).

Fixtures: ``tests/golden/grammar_programs.json``, written by
``tests/golden/make_programs.py`` from the reference's own program builders
and rewrite engine (base programs plus seeded chains of the search's
rewrites), with the reference's ``program_flops`` and input/output names.
CPU tests check that every program of a family lowers to the same kernel with
the reference's ``KERNEL_META``; GPU tests run the lowered modules against
the oracle.
"""

import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_close
from cs348k_fast_attention_grammar_b200 import grammar_backend as gb
from cs348k_fast_attention_grammar_b200.grammar_ir import (Compute, Load, ParallelLoop,
                                                           Program, Store, program_from_json,
                                                           program_to_json)

with open(os.path.join(GOLDEN, "grammar_programs.json")) as _f:
    RECORDS = json.load(_f)
IDS = [r["name"] for r in RECORDS]


def test_fixture_covers_every_family_and_rewrites():
    kinds = {r["expect"] for r in RECORDS}
    assert {"attention", "mlp_ln", "mlp", "layer_norm", "unsupported"} <= kinds
    rewritten = [r for r in RECORDS if r["chain"]]
    labels = {lab.split("(")[0] for r in rewritten for lab in r["chain"]}
    assert {"merge", "subtile", "reorder", "hoist", "sink", "unwrap"} <= labels
    assert all(r["emit_ok"] for r in RECORDS)


@pytest.mark.parametrize("rec", RECORDS, ids=IDS)
def test_json_round_trip(rec):
    prog = program_from_json(rec["program"])
    assert program_to_json(prog) == rec["program"]


@pytest.mark.parametrize("rec", RECORDS, ids=IDS)
def test_lowering_matches_reference_meta(rec):
    prog = program_from_json(rec["program"])
    if rec["expect"] == "unsupported":
        with pytest.raises(gb.UnsupportedProgram):
            gb.lower(prog)
        return
    mod = gb.lower(prog)
    assert mod.kind == rec["expect"]
    meta = mod.KERNEL_META
    assert [name for name, _ in meta["inputs"]] == rec["inputs"]
    assert meta["output"][0] == rec["outputs"][0]
    assert meta["flops"] == rec["flops"] and meta["flops_exact"] == rec["flops_exact"]
    for name, dims in meta["inputs"]:
        assert tuple(dims) == tuple(rec["program"]["tensors"][name])


@pytest.mark.parametrize("rec", [r for r in RECORDS if r["expect"] != "unsupported"],
                         ids=[r["name"] for r in RECORDS if r["expect"] != "unsupported"])
def test_emitted_source_defines_fn_and_meta(rec):
    prog = program_from_json(rec["program"])
    src = gb.emit_module(prog)
    ns = {}
    exec(compile(src, f"<{rec['name']}>", "exec"), ns)
    assert ns["KERNEL_META"] == gb.lower(prog).KERNEL_META
    code = ns["fn"].__code__
    assert list(code.co_varnames[:code.co_argcount]) == rec["inputs"]


def test_attention_scale_and_parameters():
    rec = next(r for r in RECORDS if r["name"] == "attn_N512_d64")
    mod = gb.lower(program_from_json(rec["program"]))
    assert mod.roles == {"q": "Q", "kt": "KT", "v": "V"}
    assert abs(mod.params["scale"] - 64 ** -0.5) < 1e-12
    rec = next(r for r in RECORDS if r["name"] == "mlp_ln_B64_Dm64_H128")
    mod = gb.lower(program_from_json(rec["program"]))
    assert mod.roles == {"x": "X", "w1": "W1", "w2": "W2"}
    assert abs(mod.params["eps"] - 1e-5) < 1e-12


def _gemm_prog(op_after=None, M=128, K=64, N=128):
    A = Load("A", ["m", "k"]); B = Load("B", ["k", "n"])
    c = Compute("matmul", [A, B])
    body = [A, B, c]
    out = c
    if op_after is not None:
        out = Compute(op_after, [c])
        body.append(out)
    body.append(Store("C", out, ["m", "n"]))
    return Program({"A": (M, K), "B": (K, N), "C": (M, N)},
                   [ParallelLoop("C", (M, N), ("m", "n"), body)])


def test_gemm_rules_and_rejections():
    assert gb.lower(_gemm_prog()).kind == "gemm_act"
    mod = gb.lower(_gemm_prog("relu"))
    assert mod.kind == "gemm_act" and mod.params["act"] == "relu"
    with pytest.raises(gb.UnsupportedProgram):
        gb.lower(_gemm_prog("exp"))             # exp(A @ B): no kernel
    with pytest.raises(gb.UnsupportedProgram):
        gb.lower(_gemm_prog(K=96))              # K not a multiple of 64
    with pytest.raises(gb.UnsupportedProgram):
        gb.lower(_gemm_prog("tanh"))            # op without a rule


# ---------------------------------------------------------------------------
# GPU: the lowered modules compute what the programs say
# ---------------------------------------------------------------------------
def _ln_np(r, eps):
    r = np.asarray(r, dtype=np.float64)
    return (r - r.mean(1, keepdims=True)) / np.sqrt(r.var(1, keepdims=True) + eps)


def _bf(a):
    return torch.from_numpy(a).to(torch.bfloat16).double().numpy()


GPU_RECORDS = [r for r in RECORDS if r["expect"] != "unsupported"]


@pytest.mark.gpu
@pytest.mark.parametrize("rec", GPU_RECORDS, ids=[r["name"] for r in GPU_RECORDS])
def test_lowered_module_matches_oracle(rec):
    import oracle
    from oracle.mlp import round_to_bf16
    prog = program_from_json(rec["program"])
    mod = gb.lower(prog)
    rng = np.random.default_rng(5)
    ins = {}
    for name, dims in mod.KERNEL_META["inputs"]:
        std = 1.0 if mod.kind in ("attention", "layer_norm") or name in ("X",) else dims[0] ** -0.5
        ins[name] = (rng.standard_normal(dims) * std).astype(np.float32)
    args = [torch.from_numpy(ins[n]).cuda() for n, _ in mod.KERNEL_META["inputs"]]
    out = mod.fn(*args)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    got = out.cpu().numpy()
    r = mod.roles
    if mod.kind == "attention":
        q, kt, v = (_bf(ins[r[x]]) for x in ("q", "kt", "v"))
        ref = oracle.attention(q[None, None], kt.T[None, None], v[None, None],
                               scale=mod.params["scale"])[0, 0]
        assert_close(got, ref, what=rec["name"])
    elif mod.kind == "mlp_ln":
        x, w1, w2 = (_bf(ins[r[n]]) for n in ("x", "w1", "w2"))
        h = round_to_bf16(np.maximum(x @ w1, 0)).astype(np.float64)
        res = round_to_bf16(h @ w2 + x).astype(np.float64)
        assert_close(got, _ln_np(res, mod.params["eps"]), what=rec["name"])
    elif mod.kind == "mlp":
        x, w1, w2 = (_bf(ins[r[n]]) for n in ("x", "w1", "w2"))
        ref = oracle.mlp(x, w1, w2, act=mod.params["act"], round_hidden_bf16=True)
        assert_close(got, ref, what=rec["name"])
    elif mod.kind == "layer_norm":
        assert_close(got, _ln_np(_bf(ins[r["x"]]), mod.params["eps"]), what=rec["name"])
    else:
        raise AssertionError(mod.kind)
