"""CPU oracle for the attention / MLP hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy (fp32 or fp64), the arithmetic that the
reference (nriedman/cs348k-fast-attention-grammar) defines for the hot path:

* ``attention``   -- softmax(Q K^T / sqrt(d)) V per (batch, head) pair, the
                     correct formula of ``run_attention_search.py:176-180``
                     and ``test_renderer.py:512-523``, plus an optional
                     lower-triangular (causal) mask that the reference lacks;
* ``mlp``         -- act(X W1) W2 (the GEMM -> activation -> GEMM core of
                     ``run_mlp_search.py:58-69``) with ReLU or tanh-GELU,
                     and the full reference block (ReLU, residual, LayerNorm,
                     ``run_mlp_search.py:71-93,138-149``).

It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` and
``--impl reference`` legs) may import it.  The product path in
``cs348k_fast_attention_grammar_b200`` never calls into this package.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Python
pipeline in this container (its emitted cuTile attention/MLP programs through
the reference's numpy stand-in for ``cuda.tile``, its ``flash-attn2-sota.py``
module on CPU torch) and stores inputs and outputs under ``tests/golden/``;
``tests/test_oracle.py`` checks this oracle against every stored vector.
The tanh-GELU variant has no reference counterpart (the reference MLP uses
ReLU); it is checked against ``torch.nn.functional.gelu(approximate="tanh")``.
"""

from .attention import (  # noqa: F401
    attention,
    attention_pair,
    naive_torch_pair,
    naive_fn,
    naive_fn_shipped,
    attention_flops,
    program_flops_attention,
)
from .mlp import mlp, mlp_ln_block, gelu_tanh, mlp_flops  # noqa: F401
