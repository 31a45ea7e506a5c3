"""MLP oracle (numpy) -- test infrastructure, never the product path.

The reference's MLP problem (``run_mlp_search.py:42-127``) is::

    h = X @ W1            (X [B, Dm], W1 [Dm, H], row-major)      :58-60
    a = relu(h)                                                   :62-64
    y = a @ W2            (W2 [H, Dm])                            :66-69
    r = y + X                                                     :71-74
    out = (r - mean) / sqrt(var + eps)  over Dm                   :76-93

with its oracle at ``run_mlp_search.py:138-149``.  The B200 hot path computes
the GEMM -> activation -> GEMM core ``Y = act(X W1) W2`` with ``act`` either
ReLU (the reference's) or tanh-approximate GELU (the benchmark config's).
"""

from __future__ import annotations

import math

import numpy as np


def gelu_tanh(x):
    """0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the tanh approximation
    that ``torch.nn.functional.gelu(approximate="tanh")`` implements."""
    c = math.sqrt(2.0 / math.pi)
    return 0.5 * x * (1.0 + np.tanh(c * (x + 0.044715 * x * x * x)))


def _act(h, act: str):
    if act == "gelu_tanh":
        return gelu_tanh(h)
    if act == "relu":
        return np.maximum(h, 0.0)               # run_mlp_search.py:62-64
    raise ValueError(f"unknown activation {act!r}")


def mlp(x, w1, w2, act: str = "gelu_tanh", dtype=np.float64,
        round_hidden_bf16: bool = False):
    """``act(x @ w1) @ w2`` in ``dtype``.

    ``round_hidden_bf16`` rounds the activation to bf16 before the second
    GEMM, which is what a bf16 hidden buffer holds; tests use it to separate
    kernel error from the unavoidable rounding of the stored hidden tensor.
    """
    x = np.asarray(x, dtype=dtype)
    w1 = np.asarray(w1, dtype=dtype)
    w2 = np.asarray(w2, dtype=dtype)
    h = _act(x @ w1, act)
    if round_hidden_bf16:
        h = round_to_bf16(h).astype(dtype)
    return h @ w2


def mlp_ln_block(x, w1, w2, eps: float = 1e-5, dtype=np.float64):
    """The full reference block ``LayerNorm(relu(x W1) W2 + x)`` without
    affine parameters, as ``run_mlp_search.py:138-149`` checks it."""
    x = np.asarray(x, dtype=dtype)
    y = mlp(x, w1, w2, act="relu", dtype=dtype)
    r = y + x
    mean = r.mean(axis=1, keepdims=True)
    var = r.var(axis=1, keepdims=True)
    return (r - mean) / np.sqrt(var + eps)


def round_to_bf16(a):
    """Round-to-nearest-even of float32 values to bfloat16, returned as
    float32 (bit manipulation on the IEEE encoding; NaN kept quiet)."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    r = r.astype(np.uint32)
    nan = np.isnan(a)
    r[nan] = 0x7FC00000
    return r.view(np.float32)


def mlp_flops(M: int, K: int, N: int) -> int:
    """Two GEMMs of ``2*M*K*N`` each; the activation is not counted."""
    return 4 * M * K * N
