"""Small, self-contained runs of one kernel for profilers (Nsight Compute).

    python -m cs348k_fast_attention_grammar_b200.profile_case --config cfg2 --pairs 32
    python -m cs348k_fast_attention_grammar_b200.profile_case --config cfg3 --rows 2048
    python -m cs348k_fast_attention_grammar_b200.profile_case --config ln --rows 16384

Attention: the first ``--pairs`` (batch, head) pairs of a BASELINE config at
its full S and D (the same kernel, fewer pairs per launch); MLP: the first
``--rows`` rows of X with the config's full weights; ``ln``: the row
LayerNorm on ``--rows`` rows of cfg3's feature width (4096).  Inputs are generated
before the launches; ``--iters`` launches follow (so ``ncu -s 1 -c 1`` skips
a cold first launch).  Prints the CUDA-event time per launch.
"""

from __future__ import annotations

import argparse

import torch

from .inputs import ATTN_CONFIGS, MLP_CONFIGS, make_mlp, make_qkv
from .operators import attention, gemm_act, layer_norm_rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="cfg2",
                    choices=sorted(list(ATTN_CONFIGS) + list(MLP_CONFIGS) + ["ln"]))
    ap.add_argument("--pairs", type=int, default=32)
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if a.config in ATTN_CONFIGS:
        cfg = ATTN_CONFIGS[a.config]
        q, k, v = make_qkv(cfg, range(a.pairs), dev)
        o = torch.empty_like(q)
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(a.iters):
            attention(q, k, v, causal=cfg["causal"], out=o)
        ev[1].record()
        what = f"attention {a.config} pairs={a.pairs} S={cfg['S']} D={cfg['D']}"
    elif a.config == "ln":
        K = MLP_CONFIGS["cfg3"]["K"]
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn((a.rows, K), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(a.iters):
            layer_norm_rows(x, out=y)
        ev[1].record()
        what = f"layer_norm rows={a.rows} N={K}"
    else:
        cfg = dict(MLP_CONFIGS[a.config], M=a.rows)
        x, w1, w2 = make_mlp(cfg, dev)
        h = torch.empty((a.rows, cfg["N"]), dtype=torch.bfloat16, device=dev)
        y = torch.empty((a.rows, cfg["K"]), dtype=torch.bfloat16, device=dev)
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(a.iters):
            gemm_act(x, w1, act="gelu_tanh", out=h)
            gemm_act(h, w2, act="none", out=y)
        ev[1].record()
        what = f"mlp {a.config} rows={a.rows} K={cfg['K']} N={cfg['N']}"
    torch.cuda.synchronize()
    print(f"{what}: {ev[0].elapsed_time(ev[1]) / a.iters:.4f} ms per iteration")


if __name__ == "__main__":
    main()
