#!/usr/bin/env python3
"""Fit the polynomial used by the kernel's FMA-pipe exp2 (poly_exp2_x2 in
tpsa_kernel.cu).

Method: Cody-Waite style range reduction x = n + f with n = round(x),
f in [-1/2, 1/2], so 2^x = 2^n * 2^f; 2^f is approximated by a polynomial
p(f) whose maximum *relative* error on [-1/2, 1/2] is minimised with the
Remez exchange algorithm (equioscillation on degree + 2 reference points).
The constant term is left free (p(0) != 1 exactly) because the minimax fit
trades it for a smaller worst-case error.

Prints the coefficients (highest degree first, fp32-rounded) and the fp32
evaluation error.  Usage: python fit_exp2_poly.py [degree]
"""

from __future__ import annotations

import sys

import numpy as np


def remez_relative(degree: int, lo: float = -0.5, hi: float = 0.5, iters: int = 60) -> np.ndarray:
    """Minimax coefficients c0..cd of p(f) ~ 2^f under relative error."""
    n = degree + 2
    # Chebyshev extrema as the initial reference set.
    k = np.arange(n)
    ref = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * (n - 1 - k) / (n - 1))
    dense = np.linspace(lo, hi, 200001)
    coef = None
    for _ in range(iters):
        # Solve p(x_i) - 2^x_i = (-1)^i E 2^x_i for c and E.
        a = np.zeros((n, n))
        for j in range(degree + 1):
            a[:, j] = ref ** j
        a[:, degree + 1] = ((-1.0) ** k) * np.exp2(ref)
        sol = np.linalg.solve(a, np.exp2(ref))
        coef = sol[:degree + 1]
        err = np.polynomial.polynomial.polyval(dense, coef) / np.exp2(dense) - 1.0
        # New reference: the extremum of each sign-alternating segment.
        sign = np.sign(err)
        idx = np.nonzero(np.diff(sign))[0]
        bounds = np.concatenate(([0], idx + 1, [dense.size]))
        extrema = [b0 + int(np.argmax(np.abs(err[b0:b1]))) for b0, b1 in zip(bounds[:-1], bounds[1:])]
        if len(extrema) < n:
            break
        # Keep the n consecutive extrema with the largest minimum magnitude.
        best = max(range(len(extrema) - n + 1),
                   key=lambda s: np.min(np.abs(err[extrema[s:s + n]])))
        new_ref = dense[extrema[best:best + n]]
        if np.allclose(new_ref, ref, atol=1e-12, rtol=0):
            break
        ref = new_ref
    return coef


def main() -> None:
    degree = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c = remez_relative(degree)
    c32 = c.astype(np.float32)
    f = np.linspace(-0.5, 0.5, 400001, dtype=np.float32)
    p = np.zeros_like(f)
    for ci in c32[::-1]:  # Horner in fp32, highest degree first
        p = p * f + ci
    rel = np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)
    print(f"degree {degree}, max relative error {rel.max():.3e}")
    print("coefficients, highest degree first:")
    for ci in c32[::-1]:
        print(f"  {float(ci)!r}f  ({np.float32(ci).view(np.uint32):#010x})")


if __name__ == "__main__":
    main()
