"""Generate the golden vectors under tests/golden/ from the reference itself.

Run in a container where the reference checkout is present (it is not on the
GPU box; the .npz files it writes are committed)::

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

What it runs -- all of it the reference's own code, on CPU:

* ``run_attention_search.build_attention`` (``run_attention_search.py:34-114``)
  -> ``grammar.kernel_ast.emit_module`` -> the emitted module executed through
  the reference's numpy stand-in for ``cuda.tile``/``cupy``
  (``test_renderer.py:60-123``, ``setup_backend("cpu")``);
* the search's best shipped kernel ``runs/attn_full/kernels/best_it24.py``
  (6 tiled kernels) through the same stand-in;
* ``flash-attn2-sota.py`` ``fn(K, Q, V)`` (torch SDPA on CPU), and torch SDPA
  with ``is_causal=True`` -- the call that module makes, with the flag the
  reference leaves off -- for causal pins;
* ``pytorch-naive.py`` ``fn(KT, Q, V)`` as shipped (numerically wrong; kept
  to document that);
* ``run_mlp_search.build_mlp_ln`` (``run_mlp_search.py:42-127``) and a
  GEMM -> ReLU -> GEMM program built from the same grammar nodes, through the
  stand-in.

Inputs follow the reference's own seeding where it has one
(``cp.random.RandomState(1)`` standard normal fp32, ``run_attention_search.py:173``)
and are rounded to bf16 values before the reference runs, so its fp32 output
is the exact-arithmetic target for a bf16-input kernel on the same inputs.
"""

from __future__ import annotations

import argparse
import importlib.util
import math
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_file(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _import_source(src: str, name: str):
    fd, path = tempfile.mkstemp(suffix=".py", prefix="golden_")
    with os.fdopen(fd, "w") as f:
        f.write(src)
    try:
        return _import_file(path, name)
    finally:
        os.unlink(path)


def _bf16(a):
    """Round an fp32 array to the nearest bf16 value (kept as fp32), so the
    reference computes on exactly the inputs a bf16 kernel receives."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(
        torch.bfloat16).float().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    ref = os.path.abspath(args.reference)
    sys.path.insert(0, ref)

    import test_renderer as tr                       # reference test module
    tr.setup_backend("cpu")                          # numpy cuda.tile / cupy stand-in
    import torch
    import run_attention_search as ras
    import run_mlp_search as rms
    from grammar.kernel_ast import (Program, ParallelLoop, Load, Store,
                                    Compute, emit_module)

    out = {}

    # --- 1. attention through the reference's emitted 8-stage program --------
    for (N, d, tile, sub) in [(512, 64, None, None), (256, 128, 64, 32),
                              (128, 64, 32, 16)]:
        prog = ras.build_attention(N, d, tile=tile, subtile_k=sub)
        mod = _import_source(emit_module(prog), f"attn_{N}_{d}")
        rng = np.random.RandomState(1)               # run_attention_search.py:173
        ins = {nm: _bf16(rng.randn(*s)) for nm, s in mod.KERNEL_META["inputs"]}
        o = np.asarray(mod.fn(*[ins[nm] for nm, _ in mod.KERNEL_META["inputs"]]))
        key = f"attn_program_N{N}_d{d}"
        out[key] = dict(KT=ins["KT"], Q=ins["Q"], V=ins["V"], O=o.astype(np.float32),
                        flops=np.int64(mod.KERNEL_META["flops"]))
        print(key, o.shape, "flops", mod.KERNEL_META["flops"])

    # --- 2. the search's best shipped kernel (6 tiled kernels) -----------------
    best = _import_file(os.path.join(ref, "runs/attn_full/kernels/best_it24.py"),
                        "best_it24")
    rng = np.random.RandomState(2)
    ins = {nm: _bf16(rng.randn(*s)) for nm, s in best.KERNEL_META["inputs"]}
    o = np.asarray(best.fn(*[ins[nm] for nm, _ in best.KERNEL_META["inputs"]]))
    out["attn_best_it24_N512_d64"] = dict(KT=ins["KT"], Q=ins["Q"], V=ins["V"],
                                          O=o.astype(np.float32))
    print("best_it24", o.shape)

    # --- 3. flash-attn2-sota.py fn(K, Q, V) and its causal flag ----------------
    sota = _import_file(os.path.join(ref, "flash-attn2-sota.py"), "sota")
    g = torch.Generator().manual_seed(3)
    shp = sota.KERNEL_META["inputs"][0][1]           # [1, 1, 512, 64]
    K = torch.randn(shp, generator=g).bfloat16().float()
    Q = torch.randn(shp, generator=g).bfloat16().float()
    V = torch.randn(shp, generator=g).bfloat16().float()
    o = sota.fn(K, Q, V)
    out["sdpa_N512_d64"] = dict(K=K.numpy(), Q=Q.numpy(), V=V.numpy(), O=o.numpy())
    # causal: the same torch call the module makes, with is_causal=True
    for (S, D, seed) in [(384, 128, 4), (200, 64, 5)]:
        g = torch.Generator().manual_seed(seed)
        q, k, v = (torch.randn(1, 1, S, D, generator=g).bfloat16().float() for _ in range(3))
        oc = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        out[f"sdpa_causal_S{S}_d{D}"] = dict(Q=q.numpy(), K=k.numpy(), V=v.numpy(),
                                             O=oc.numpy())
    print("sdpa done")

    # --- 4. pytorch-naive.py as shipped ----------------------------------------
    naive = _import_file(os.path.join(ref, "pytorch-naive.py"), "naive")
    rng = np.random.RandomState(0)
    ins = {nm: rng.randn(*s).astype(np.float32) for nm, s in naive.KERNEL_META["inputs"]}
    o = naive.fn(*[torch.from_numpy(ins[nm]) for nm, _ in naive.KERNEL_META["inputs"]])
    out["naive_shipped_N512_d64"] = dict(KT=ins["KT"], Q=ins["Q"], V=ins["V"],
                                         O=o.numpy().astype(np.float32))

    # --- 5. MLP: the reference block and the GEMM-ReLU-GEMM core ---------------
    B, Dm, Hd = 64, 64, 128
    prog = rms.build_mlp_ln(B, Dm, Hd)
    mod = _import_source(emit_module(prog), "mlp_ln")
    rng = np.random.RandomState(1)                   # run_mlp_search.py:141
    ins = {nm: _bf16(rng.randn(*s)) for nm, s in mod.KERNEL_META["inputs"]}
    o = np.asarray(mod.fn(*[ins[nm] for nm, _ in mod.KERNEL_META["inputs"]]))
    out[f"mlp_ln_B{B}_Dm{Dm}_H{Hd}"] = dict(X=ins["X"], W1=ins["W1"], W2=ins["W2"],
                                            O=o.astype(np.float32))

    # GEMM -> relu -> GEMM, stages h, a, y exactly as build_mlp_ln writes them
    X = Load("X", ["b", "dm"]); W1 = Load("W1", ["dm", "hid"])
    h = Compute("matmul", [X, W1])
    s_h = ParallelLoop("h", (B, Hd), ("b", "hid"), [X, W1, h, Store("h", h, ["b", "hid"])])
    hL = Load("h", ["b", "hid"]); a = Compute("relu", [hL])
    s_a = ParallelLoop("a", (B, Hd), ("b", "hid"), [hL, a, Store("a", a, ["b", "hid"])])
    aL = Load("a", ["b", "hid"]); W2 = Load("W2", ["hid", "dm"])
    y = Compute("matmul", [aL, W2])
    s_y = ParallelLoop("y", (B, Dm), ("b", "dm"), [aL, W2, y, Store("y", y, ["b", "dm"])])
    core = Program({"X": (B, Dm), "W1": (Dm, Hd), "W2": (Hd, Dm), "h": (B, Hd),
                    "a": (B, Hd), "y": (B, Dm)}, [s_h, s_a, s_y])
    mod = _import_source(emit_module(core), "mlp_core")
    rng = np.random.RandomState(7)
    ins = {nm: _bf16(rng.randn(*s) / math.sqrt(s[0] if nm != "X" else 1))
           for nm, s in mod.KERNEL_META["inputs"]}
    o = np.asarray(mod.fn(*[ins[nm] for nm, _ in mod.KERNEL_META["inputs"]]))
    out[f"mlp_relu_core_B{B}_Dm{Dm}_H{Hd}"] = dict(X=ins["X"], W1=ins["W1"],
                                                   W2=ins["W2"], O=o.astype(np.float32))
    print("mlp done")

    for key, arrs in out.items():
        np.savez_compressed(os.path.join(args.out, key + ".npz"), **arrs)
    print("wrote", len(out), "fixtures to", args.out)


if __name__ == "__main__":
    main()
