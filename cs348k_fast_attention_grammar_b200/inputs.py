"""Seeded synthetic inputs for the benchmark configurations.

No dataset is involved: the reference's own harness draws standard-normal
inputs (``bench.py:45-46``; ``run_attention_search.py:173``).  Here every
(batch, head) pair's Q, K and V come from a counter-based generator (torch's
Philox) keyed on ``(seed, tensor, pair)``, so any sharding of the pairs over
ranks reproduces bit-identical tensors and a checker can regenerate any single
pair on its own.
"""

from __future__ import annotations

import math

import torch

MASK64 = (1 << 64) - 1
TENSOR_IDS = {"q": 1, "k": 2, "v": 3, "x": 4, "w1": 5, "w2": 6}

# BASELINE configurations (attention: B, H, S, D, causal, seed, value scale).
ATTN_CONFIGS = {
    "cfg0": dict(B=1, H=4, S=256, D=64, causal=False, seed=0, amp=1.0),
    "cfg1": dict(B=8, H=16, S=4096, D=64, causal=False, seed=1, amp=1.0),
    "cfg2": dict(B=4, H=32, S=8192, D=128, causal=True, seed=2, amp=0.5),
    "cfg4": dict(B=64, H=32, S=16384, D=128, causal=True, seed=4, amp=0.5),
}
MLP_CONFIGS = {
    "cfg3": dict(M=8192, K=4096, N=16384, seed=3),
}


def _splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return (x ^ (x >> 31)) & MASK64


def pair_seed(seed: int, tensor: str, pair: int) -> int:
    """63-bit generator seed for one tensor of one (batch, head) pair."""
    x = _splitmix64(seed & MASK64)
    x = _splitmix64(x ^ TENSOR_IDS[tensor])
    x = _splitmix64(x ^ (pair & MASK64))
    return x & ((1 << 63) - 1)


def pair_tensor(seed: int, tensor: str, pair: int, S: int, D: int, amp: float,
                device, dtype=torch.bfloat16) -> torch.Tensor:
    """``amp * N(0, 1)`` of shape ``[S, D]`` for one pair, rounded to ``dtype``."""
    g = torch.Generator(device=device)
    g.manual_seed(pair_seed(seed, tensor, pair))
    t = torch.randn((S, D), generator=g, device=device, dtype=torch.float32)
    if amp != 1.0:
        t.mul_(amp)
    return t.to(dtype)


def make_qkv(cfg: dict, pairs, device, dtype=torch.bfloat16):
    """Q, K, V for the listed flattened pairs ``p = b*H + h`` as
    ``[1, len(pairs), S, D]`` tensors (a shard viewed as one batch)."""
    pairs = list(pairs)
    S, D = cfg["S"], cfg["D"]
    out = []
    for name in ("q", "k", "v"):
        t = torch.empty((1, len(pairs), S, D), dtype=dtype, device=device)
        for i, p in enumerate(pairs):
            t[0, i].copy_(pair_tensor(cfg["seed"], name, p, S, D, cfg["amp"], device, dtype))
        out.append(t)
    return tuple(out)


def make_mlp(cfg: dict, device, dtype=torch.bfloat16):
    """X ~ N(0, 1), W1 ~ N(0, 1/K), W2 ~ N(0, 1/N) (fan-in scaling)."""
    M, K, N, seed = cfg["M"], cfg["K"], cfg["N"], cfg["seed"]
    g = torch.Generator(device=device)
    g.manual_seed(pair_seed(seed, "x", 0))
    x = torch.randn((M, K), generator=g, device=device).to(dtype)
    g.manual_seed(pair_seed(seed, "w1", 0))
    w1 = (torch.randn((K, N), generator=g, device=device) / math.sqrt(K)).to(dtype)
    g.manual_seed(pair_seed(seed, "w2", 0))
    w2 = (torch.randn((N, K), generator=g, device=device) / math.sqrt(N)).to(dtype)
    return x, w1, w2
