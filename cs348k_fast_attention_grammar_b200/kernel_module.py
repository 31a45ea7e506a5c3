"""The reference's kernel-module protocol (``bench.py:14-20``) over the B200
kernels, so the reference's own harness can time this library unmodified::

    python bench.py --kernel <this file> --dtype fp32       (reference bench)

A module exposes ``fn(*inputs) -> output`` with inputs in sorted tensor-name
order (``grammar/kernel_ast.py:673``) and ``KERNEL_META`` (``:1280-1287``).
The reference's arrays are DLPack-capable (cupy); they are wrapped with
``torch.from_dlpack`` as ``pytorch-naive.py:36-38`` does.  fp16 and bf16
arrays run the tensor cores in their own type (fp32 accumulate); fp32 arrays
(the reference's default) are staged on the device in the same C call as
bf16 hi + lo pairs whose three significant products the GEMMs accumulate
(about 16 significant bits), with an fp32 result.  As in the reference, the
callee allocates and returns the output.
"""

from __future__ import annotations

import torch

from .operators import attention, attention_f32

N, D = 512, 64

# program_flops of the reference's 8-stage attention program at N=512, d=64
# (grammar/kernel_ast.py:1110-1147): 4*N^2*d + 6*N^2.
KERNEL_META = {
    "inputs": [["KT", [D, N]], ["Q", [N, D]], ["V", [N, D]]],
    "output": ["O", [N, D]],
    "flops": 4 * N * N * D + 6 * N * N,
    "flops_exact": True,
}

# flash-attn2-sota.py:65 -- fn(K, Q, V) on [1, 1, 512, 64]
SOTA_KERNEL_META = {
    "inputs": [["K", [1, 1, N, D]], ["Q", [1, 1, N, D]], ["V", [1, 1, N, D]]],
    "output": ["O", [1, 1, N, D]],
    "flops": 4 * N * N * D + 6 * N * N,
    "flops_exact": True,
}


def _as_torch(x) -> torch.Tensor:
    return x if isinstance(x, torch.Tensor) else torch.from_dlpack(x)


def fn(KT, Q, V):
    """``fn(KT, Q, V) -> O`` for ``KT [d, N]``, ``Q [N, d]``, ``V [N, d]``
    (the signature of ``pytorch-naive.py:23`` and every emitted module).
    fp32 inputs go through one C call (device-side hi/lo staging, fp32
    output; head dims above 64 fall back to plain bf16 staging); bf16 and fp16
    inputs through the batched operator, in their own type."""
    KT, Q, V = _as_torch(KT), _as_torch(Q), _as_torch(V)
    if Q.dtype == torch.float32:
        return attention_f32(Q.contiguous(), KT.contiguous(), V.contiguous(), k_transposed=True,
                             precise=Q.shape[1] <= 64)
    # bf16 / fp16: K must be contiguous along d, so KT [d, N] is transposed once.
    q = Q.contiguous().unsqueeze(0).unsqueeze(0)
    k = KT.t().contiguous().unsqueeze(0).unsqueeze(0)
    v = V.contiguous().unsqueeze(0).unsqueeze(0)
    return attention(q, k, v, causal=False)[0, 0]


def sota_fn(K, Q, V):
    """``fn(K, Q, V)`` on ``[B, H, S, D]`` tensors, the argument order of
    ``flash-attn2-sota.py:41``."""
    K, Q, V = _as_torch(K), _as_torch(Q), _as_torch(V)
    precise = Q.dtype == torch.float32 and Q.shape[-1] <= 64
    return attention(Q.contiguous(), K.contiguous(), V.contiguous(), causal=False,
                     precise=precise)
