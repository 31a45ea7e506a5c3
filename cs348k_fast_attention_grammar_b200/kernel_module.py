"""The reference's kernel-module protocol (``bench.py:14-20``) over the B200
kernels, so the reference's own harness can time this library unmodified::

    python bench.py --kernel <this file> --dtype fp32       (reference bench)

A module exposes ``fn(*inputs) -> output`` with inputs in sorted tensor-name
order (``grammar/kernel_ast.py:673``) and ``KERNEL_META`` (``:1280-1287``).
The reference's arrays are DLPack-capable (cupy); they are wrapped with
``torch.from_dlpack`` as ``pytorch-naive.py:36-38`` does, cast to bf16 for the
tensor cores (fp32 accumulate), and the result is returned in the input dtype.
As in the reference, the callee allocates and returns the output.
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
    fp32 inputs go through one C call (device-side bf16 staging, fp32 output);
    bf16 inputs through the batched operator."""
    KT, Q, V = _as_torch(KT), _as_torch(Q), _as_torch(V)
    if Q.dtype == torch.float32:
        return attention_f32(Q.contiguous(), KT.contiguous(), V.contiguous(), k_transposed=True)
    dtype = Q.dtype
    q = Q.to(torch.bfloat16).unsqueeze(0).unsqueeze(0)
    k = KT.t().to(torch.bfloat16).contiguous().unsqueeze(0).unsqueeze(0)
    v = V.to(torch.bfloat16).contiguous().unsqueeze(0).unsqueeze(0)
    o = attention(q.contiguous(), k, v, causal=False)
    return o[0, 0].to(dtype)


def sota_fn(K, Q, V):
    """``fn(K, Q, V)`` on ``[B, H, S, D]`` tensors, the argument order of
    ``flash-attn2-sota.py:41``."""
    K, Q, V = _as_torch(K), _as_torch(Q), _as_torch(V)
    if Q.dtype == torch.float32 and Q.shape[0] == 1 and Q.shape[1] == 1:
        o = attention_f32(Q[0, 0].contiguous(), K[0, 0].contiguous(), V[0, 0].contiguous())
        return o.view(Q.shape)
    dtype = Q.dtype
    bf = torch.bfloat16
    o = attention(Q.to(bf).contiguous(), K.to(bf).contiguous(), V.to(bf).contiguous(),
                  causal=False)
    return o.to(dtype)
