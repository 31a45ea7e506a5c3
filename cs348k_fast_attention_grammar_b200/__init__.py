"""B200-native (sm_100a) fused attention forward and GEMM-GELU-GEMM MLP.

Public operators (all run the hand-written kernels of ``libfa_b200.so``
through its C ABI, ``include/fa_b200.h``; there is no fallback path):

    attention(q, k, v, causal=False, scale=None, out=None)   # [B, H, S, D] bf16/fp16/fp32, D 8..128
    attention_bshd(q, k, v, causal=False)                    # (B, S, H, D) layout
    attention_f32(q, k, v, k_transposed=False)               # 2-D fp32 [N, D] (fn(KT, Q, V))
    attention_from_host(q, k, v, causal=False, ...)          # pinned host tensors
    mlp(x, w1, w2, act="gelu_tanh")                          # act(x@w1)@w2, bf16/fp16
    mlp_ln(x, w1, w2)                                        # LN(relu(x@w1)@w2 + x)
    gemm_act(a, b, act="none")                               # act(a@b)

``kernel_module`` exposes the reference's ``fn(KT, Q, V)`` + ``KERNEL_META``
protocol; ``parallel`` holds the batch x head sharding used by ``bench.py``.
"""

from ._lib import FaError, lib_path, load  # noqa: F401
from .operators import (  # noqa: F401
    attention,
    attention_bshd,
    attention_f32,
    attention_from_host,
    device_status,
    gemm_act,
    layer_norm_rows,
    mlp,
    mlp_from_host,
    mlp_ln,
)

__all__ = ["attention", "attention_bshd", "attention_f32", "attention_from_host", "mlp", "mlp_from_host", "mlp_ln",
           "layer_norm_rows", "gemm_act",
           "device_status", "FaError", "load", "lib_path"]
