"""Fit the polynomial behind the attention kernel's FMA-pipe exp2.

The softmax computes ``2^x`` for every score.  Most go to the MUFU unit
(``ex2.approx``); a fraction is computed on the FMA pipe instead, by the
textbook base-2 range reduction ``x = j + f`` (j = nearest integer, f in
[-1/2, 1/2]), ``2^x = 2^j * p(f)``, with ``2^j`` applied by adding ``j`` to the
IEEE exponent field.  ``p`` is the degree-3 polynomial minimising the maximum
*relative* error of ``p(f) / 2^f`` on [-1/2, 1/2], found here with the Remez
exchange algorithm (alternation at 5 points), then rounded to fp32.

    python -m cs348k_fast_attention_grammar_b200.fit_exp2_poly

prints the coefficients used in csrc/attn_fwd.cu and the error bound that
tests/test_exp2_poly.py checks (the probabilities are rounded to bf16, whose
relative spacing is 2^-8, so ~1e-4 is far below what the output can resolve).
"""

from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def remez(degree: int = DEGREE, iters: int = 30):
    n = degree + 2
    # Chebyshev extrema as the initial reference set
    x = 0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(LO, HI, 200001)
    c = None
    for _ in range(iters):
        # p(x_i) - 2^x_i = (-1)^i E 2^x_i   ->   [x^k ..., -(-1)^i 2^x_i] [c; E] = 2^x_i
        A = np.zeros((n, n))
        for k in range(degree + 1):
            A[:, k] = x ** k
        A[:, -1] = -((-1.0) ** np.arange(n)) * np.exp2(x)
        sol = np.linalg.solve(A, np.exp2(x))
        c = sol[:-1]
        err = np.polynomial.polynomial.polyval(grid, c) / np.exp2(grid) - 1.0
        # new reference: the extremum of |err| in each sign-constant segment
        sign_change = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate(([0], sign_change + 1, [len(grid)]))
        ext = [s + np.argmax(np.abs(err[s:e])) for s, e in zip(bounds[:-1], bounds[1:])]
        if len(ext) != n:
            break
        x = grid[ext]
    return c


def coefficients_f32():
    return np.asarray(remez(), dtype=np.float32)


def max_rel_error(c32) -> float:
    f = np.linspace(LO, HI, 200001, dtype=np.float32)
    p = np.float32(c32[3])
    for k in (2, 1, 0):
        p = p * f + np.float32(c32[k])
    return float(np.max(np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    c = coefficients_f32()
    for k, v in enumerate(c):
        print(f"c{k} = {float(v)!r:<24} ({np.float32(v).view(np.uint32):#010x})")
    print(f"max relative error on [-1/2, 1/2]: {max_rel_error(c):.3e}")
