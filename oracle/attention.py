"""Attention oracle (numpy) -- test infrastructure, never the product path.

The formula is the reference's correct one:

* ``run_attention_search.py:176-180`` (``verify``)::

      s = (Q @ KT) / sqrt(d); e = exp(s - s.max(1, keepdims=True))
      P = e / e.sum(1, keepdims=True); ref = P @ V

* ``test_renderer.py:512-523`` (``_np_softmax`` / ``_attention_ref``), the same
  math on the renderer's test cases;
* ``pytorch-naive.py:1-10`` (docstring of the shipped naive kernel: S, Ss,
  mx = rowmax, sb, e, sm = rowsum, P, O), whose code at ``:48,57`` takes a
  sum without keepdim instead of a max; ``naive_fn_shipped`` restates that
  shipped behaviour only so the tests can show it differs.

Causal masking is not in the reference.  It follows the semantics of the API
the reference times (``flash-attn2-sota.py:60``, torch
``scaled_dot_product_attention(is_causal=True)``): key j is visible to query i
iff j <= i (top-left aligned lower triangle), applied before the row max.
"""

from __future__ import annotations

import math

import numpy as np


def attention_pair(q, k, v, causal: bool = False, scale: float | None = None,
                   dtype=np.float64, row_chunk: int = 1024) -> np.ndarray:
    """softmax(q k^T * scale) v for one (batch, head) pair.

    q: [Sq, D], k: [Sk, D], v: [Sk, D] (any float dtype; promoted to ``dtype``).
    Rows are processed in chunks of ``row_chunk`` so S = 16384 stays within a
    few hundred MB.  Follows ``run_attention_search.py:176-180``.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    sq, d = q.shape
    sk = k.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    out = np.empty((sq, v.shape[1]), dtype=dtype)
    kt = k.T
    for r0 in range(0, sq, row_chunk):
        r1 = min(sq, r0 + row_chunk)
        s = (q[r0:r1] @ kt) * dtype(scale)              # S and Ss stages
        if causal:
            rows = np.arange(r0, r1)[:, None]
            cols = np.arange(sk)[None, :]
            s = np.where(cols > rows, -np.inf, s)
        mx = s.max(axis=1, keepdims=True)                # mx = rowmax(Ss)
        e = np.exp(s - mx)                               # sb, e
        p = e / e.sum(axis=1, keepdims=True)             # sm, P
        out[r0:r1] = p @ v                               # O = P @ V
    return out


def attention(q, k, v, causal: bool = False, scale: float | None = None,
              pairs=None, dtype=np.float64) -> np.ndarray:
    """Batched oracle on ``[B, H, S, D]`` arrays; returns ``[B, H, S, D]``.

    ``pairs`` optionally restricts the work to a list of flattened
    ``p = b * H + h`` indices; the other pairs of the result are NaN.
    """
    q = np.asarray(q)
    B, H, S, D = q.shape
    out = np.full((B, H, S, np.asarray(v).shape[-1]), np.nan, dtype=dtype)
    todo = range(B * H) if pairs is None else pairs
    for p in todo:
        b, h = divmod(int(p), H)
        out[b, h] = attention_pair(q[b, h], k[b, h], v[b, h], causal, scale, dtype)
    return out


def naive_fn(KT, Q, V) -> np.ndarray:
    """The reference kernel-module call ``fn(KT, Q, V) -> O`` with the correct
    math (``pytorch-naive.py:23-65`` as its docstring ``:1-10`` specifies;
    inputs in sorted-name order as ``grammar/kernel_ast.py:673`` emits)."""
    Q = np.asarray(Q, dtype=np.float32)
    KT = np.asarray(KT, dtype=np.float32)
    V = np.asarray(V, dtype=np.float32)
    scores = (Q @ KT) * np.float32(Q.shape[-1] ** -0.5)
    mx = scores.max(axis=1, keepdims=True)
    e = np.exp(scores - mx)
    P = e / e.sum(axis=1, keepdims=True)
    return P @ V


def naive_fn_shipped(KT, Q, V) -> np.ndarray:
    """What ``pytorch-naive.py:41-63`` computes as shipped: ``torch.sum`` over
    dim 1 without keepdim for both ``mx`` and ``sm`` (``:48,57``), which then
    broadcast along the key axis (``:51,60``).  Kept only to document that the
    shipped kernel is not an oracle."""
    Q = np.asarray(Q, dtype=np.float32)
    KT = np.asarray(KT, dtype=np.float32)
    V = np.asarray(V, dtype=np.float32)
    scores = (Q @ KT) * np.float32(Q.shape[-1] ** -0.5)
    mx = scores.sum(axis=1)                 # shape [N], broadcasts over columns
    e = np.exp(scores - mx)
    sm = e.sum(axis=1)
    P = e / sm
    return P @ V


def naive_torch_pair(q, k, v, causal: bool = False, row_chunk: int = 2048):
    """The correct naive restatement of ``pytorch-naive.py:41-63`` in fp32
    torch on the CPU (keepdim row max, then exp, row sum, divide), one
    (batch, head) pair of ``[S, D]`` tensors, every intermediate materialised
    per row chunk.  This is the timed CPU baseline (it uses all the threads
    torch is given) and is checked against ``attention_pair`` in the tests."""
    import torch
    q = q.float()
    k = k.float()
    v = v.float()
    S, D = q.shape
    scale = D ** -0.5
    out = torch.empty((S, v.shape[1]), dtype=torch.float32)
    for r0 in range(0, S, row_chunk):
        r1 = min(S, r0 + row_chunk)
        scores = (q[r0:r1] @ k.t()) * scale
        if causal:
            rows = torch.arange(r0, r1)[:, None]
            scores = scores.masked_fill(torch.arange(k.shape[0])[None, :] > rows,
                                        float("-inf"))
        mx = torch.amax(scores, dim=1, keepdim=True)
        e = torch.exp(scores - mx)
        sm = torch.sum(e, dim=1, keepdim=True)
        out[r0:r1] = (e / sm) @ v
    return out


def attention_flops(B: int, H: int, S: int, D: int, causal: bool) -> int:
    """Algorithmic FLOPs of the forward: ``4*B*H*S^2*D`` (the reference's
    convention, ``old/benchmark.py:131``), halved for the causal triangle."""
    f = 4 * B * H * S * S * D
    return f // 2 if causal else f


def program_flops_attention(N: int, d: int) -> int:
    """The reference's ``program_flops`` for its 8-stage attention program
    (``grammar/kernel_ast.py:1110-1147``): two matmuls ``2*N*N*d`` each plus
    six N^2 pointwise/row-reduction stages (Ss, mx, sb, e, sm, P)."""
    return 4 * N * N * d + 6 * N * N
