"""The FMA-pipe exp2 of the attention kernel: its constants are the Remez fit
of fit_exp2_poly.py, and a bit-level numpy restatement of the kernel routine
(round-to-nearest by the 1.5 * 2^23 addition, degree-3 polynomial, exponent
field add) stays within 1e-4 relative error of exp2 over the softmax range."""

import os
import re

import numpy as np

from conftest import ROOT
from cs348k_fast_attention_grammar_b200 import fit_exp2_poly

SRC = os.path.join(ROOT, "cs348k_fast_attention_grammar_b200", "csrc", "attn_fwd.cu")


def _kernel_coeffs():
    text = open(SRC).read()
    vals = {int(k): float(v) for k, v in re.findall(r"kExpC(\d)\s*=\s*([0-9.eE+-]+)f", text)}
    return np.array([vals[i] for i in range(4)], dtype=np.float32)


def _exp2_fma_f32(x):
    """numpy restatement of exp2_fma() in csrc/attn_fwd.cu, all in float32."""
    c = _kernel_coeffs()
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    j = (t - magic).astype(np.float32)
    f = (x - j).astype(np.float32)
    p = np.float32(c[3])
    for k in (2, 1, 0):
        p = (p * f + c[k]).astype(np.float32)   # fma vs mul+add: < 1 ulp apart
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.view(np.float32)


def test_kernel_constants_are_the_remez_fit():
    np.testing.assert_array_equal(_kernel_coeffs(), fit_exp2_poly.coefficients_f32())
    assert fit_exp2_poly.max_rel_error(_kernel_coeffs()) < 1e-4


def test_emulated_exp2_accuracy_over_softmax_range():
    x = np.linspace(-120.0, 8.0, 200001, dtype=np.float32)
    got = _exp2_fma_f32(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / ref - 1.0)) < 1.2e-4


def test_emulated_exp2_masked_scores_vanish():
    got = _exp2_fma_f32(np.array([-np.inf, -1e30, -200.0], dtype=np.float32))
    assert np.all(got > 0) and np.all(got < 1e-37)
