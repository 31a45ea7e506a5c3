"""Generate tests/golden/grammar_programs.json from the reference's grammar.

Run where the reference checkout is present (it is not on the GPU box; the
JSON it writes is committed)::

    python tests/golden/make_programs.py --reference <path-to-reference-checkout>

What it records -- all produced by the reference's own code on CPU:

* the programs its drivers search from: ``run_attention_search.build_attention``
  (``run_attention_search.py:34-114``) at several sizes / tilings and
  ``run_mlp_search.build_mlp_ln`` (``run_mlp_search.py:42-127``), plus a
  GEMM -> ReLU -> GEMM program and a lone LayerNorm stage built from the same
  grammar nodes;
* for each, programs reached by seeded random chains of the search's own
  rewrites (``grammar.optimization.enumerate_rewrites`` over
  ``DEFAULT_RULES``: hoist, sink, subtile_reduction, unwrap_reduction, merge,
  merge_reductions, reorder), keeping only steps whose result the reference's
  ``emit_module`` accepts -- the structures its Stage-2 search can keep;
* per program: the reference's ``program_flops`` and input/output names
  (``grammar/kernel_ast.py:1110-1147, 665-675``), and whether its own
  ``emit_module`` accepts the program.

The B200 backend must lower every accepted program of a family to the same
kernel and report the same ``KERNEL_META``.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import sys
import zlib

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "grammar_programs.json"))
    ap.add_argument("--chains", type=int, default=3)
    ap.add_argument("--depth", type=int, default=8)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    sys.path.insert(0, REPO)

    import run_attention_search as ras
    import run_mlp_search as rms
    from grammar.kernel_ast import (Program, ParallelLoop, Load, Store, Compute,
                                    emit_module, program_flops, _program_io)
    from grammar.optimization import enumerate_rewrites, DEFAULT_RULES
    from cs348k_fast_attention_grammar_b200.grammar_ir import program_to_json

    def relu_core(B, Dm, H):
        X = Load("X", ["b", "dm"]); W1 = Load("W1", ["dm", "hid"])
        h = Compute("matmul", [X, W1])
        s_h = ParallelLoop("h", (B, H), ("b", "hid"), [X, W1, h, Store("h", h, ["b", "hid"])])
        hL = Load("h", ["b", "hid"]); a = Compute("relu", [hL])
        s_a = ParallelLoop("a", (B, H), ("b", "hid"), [hL, a, Store("a", a, ["b", "hid"])])
        aL = Load("a", ["b", "hid"]); W2 = Load("W2", ["hid", "dm"])
        y = Compute("matmul", [aL, W2])
        s_y = ParallelLoop("y", (B, Dm), ("b", "dm"), [aL, W2, y, Store("y", y, ["b", "dm"])])
        return Program({"X": (B, Dm), "W1": (Dm, H), "W2": (H, Dm), "h": (B, H),
                        "a": (B, H), "y": (B, Dm)}, [s_h, s_a, s_y])

    def layer_norm_only(B, Dm, eps=1e-5):
        # the LayerNorm stage of run_mlp_search.py:76-93 on an input tensor
        rL = Load("r", ["b", "dm"]); s1 = Compute("rowsum", [rL], axis="dm")
        r2a, r2b = Load("r", ["b", "dm"]), Load("r", ["b", "dm"])
        rr = Compute("mul", [r2a, r2b]); s2 = Compute("rowsum", [rr], axis="dm")
        mean = Compute("mulc", [s1], const=1.0 / Dm)
        meansq = Compute("mulc", [s2], const=1.0 / Dm)
        mean2 = Compute("mul", [mean, mean])
        var = Compute("sub", [meansq, mean2])
        vareps = Compute("addc", [var], const=eps)
        std = Compute("sqrt", [vareps])
        r3 = Load("r", ["b", "dm"])
        centered = Compute("sub", [r3, mean])
        out = Compute("div", [centered, std])
        s_ln = ParallelLoop("out", (B, Dm), ("b", "dm"),
                            [rL, s1, r2a, r2b, rr, s2, mean, meansq, mean2, var,
                             vareps, std, r3, centered, out, Store("out", out, ["b", "dm"])])
        return Program({"r": (B, Dm), "out": (B, Dm)}, [s_ln])

    def unnormalised_attention(N, d):
        # exp(S) @ V without the softmax normalisation: no kernel computes it
        Q = Load("Q", ["i", "dd"]); KT = Load("KT", ["dd", "j"])
        S = Compute("matmul", [Q, KT])
        s_S = ParallelLoop("S", (N, N), ("i", "j"), [Q, KT, S, Store("S", S, ["i", "j"])])
        SL = Load("S", ["i", "j"]); e = Compute("exp", [SL])
        s_e = ParallelLoop("e", (N, N), ("i", "j"), [SL, e, Store("e", e, ["i", "j"])])
        eL = Load("e", ["i", "j"]); V = Load("V", ["j", "dd"]); O = Compute("matmul", [eL, V])
        s_O = ParallelLoop("O", (N, d), ("i", "dd"), [eL, V, O, Store("O", O, ["i", "dd"])])
        return Program({"Q": (N, d), "KT": (d, N), "V": (N, d), "S": (N, N), "e": (N, N),
                        "O": (N, d)}, [s_S, s_e, s_O])

    bases = [
        ("attn_N512_d64", "attention", ras.build_attention(512, 64)),
        ("attn_N256_d128_t64_k32", "attention", ras.build_attention(256, 128, tile=64, subtile_k=32)),
        ("attn_N1024_d64_t128_k64", "attention", ras.build_attention(1024, 64, tile=128, subtile_k=64)),
        ("attn_N128_d32", "attention", ras.build_attention(128, 32)),
        ("attn_N128_d256", "unsupported", ras.build_attention(128, 256)),
        ("mlp_ln_B64_Dm64_H128", "mlp_ln", rms.build_mlp_ln(64, 64, 128)),
        ("mlp_ln_B256_Dm512_H1024_t64_k64", "mlp_ln",
         rms.build_mlp_ln(256, 512, 1024, tile=64, subtile_k=64)),
        ("relu_core_B128_Dm64_H256", "mlp", relu_core(128, 64, 256)),
        ("layer_norm_B100_Dm512", "layer_norm", layer_norm_only(100, 512)),
        ("unnormalised_attn_N256_d64", "unsupported", unnormalised_attention(256, 64)),
    ]

    def emits(prog):
        try:
            emit_module(prog)
            return True
        except Exception:
            return False

    def record(name, expect, prog, chain):
        emit_ok = emits(prog)
        flops, exact = program_flops(prog)
        inputs, _inter, outputs = _program_io(prog)
        return {"name": name, "expect": expect, "chain": chain, "emit_ok": emit_ok,
                "flops": int(flops), "flops_exact": bool(exact), "inputs": inputs,
                "outputs": outputs, "program": program_to_json(prog)}

    out = []
    for name, expect, prog in bases:
        out.append(record(name, expect, prog, []))
        if expect == "unsupported":
            continue
        for c in range(args.chains):
            rng = random.Random(zlib.crc32(name.encode()) + 17 * c)
            cur, chain = prog, []
            for step in range(args.depth):
                rws = enumerate_rewrites(cur, DEFAULT_RULES)
                rng.shuffle(rws)
                for rw in rws:
                    cand = rw.resolve(cur)
                    # keep only structures the reference itself can emit (the
                    # search scores the others inf and never keeps them)
                    if cand is not None and emits(cand):
                        cur = cand
                        chain.append(rw.label)
                        break
                else:
                    break
            out.append(record(f"{name}/chain{c}", expect, cur, chain))
    with open(args.out, "w") as f:
        json.dump(out, f, indent=None, separators=(",", ":"))
    for r in out:
        print(f"{r['name']:44s} {r['expect']:12s} emit_ok={r['emit_ok']} flops={r['flops']} "
              f"chain={r['chain']}")
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
