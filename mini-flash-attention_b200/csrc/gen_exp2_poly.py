"""Derive the exp2 polynomial used by the softmax warps (build-time helper; the output is
pasted into csrc/mfa_exp2.cuh, and tests/test_exp2_poly.py re-runs the derivation).

Method (classic Cody-Waite range reduction + Remez minimax, nothing taken from any
library): 2^x = 2^j * 2^f with j = round-to-nearest(x) and f = x - j in [-1/2, 1/2]. The
polynomial p(f) = c0 + c1 f + c2 f^2 + c3 f^3 minimises max |p(f) / 2^f - 1| on [-1/2, 1/2];
it is found with the Remez exchange algorithm on the relative error (weight 2^-f), then
rounded to float32.
"""
from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def remez(degree: int = DEGREE, iters: int = 60) -> np.ndarray:
    n = degree + 2
    # Chebyshev-like initial reference points
    k = np.arange(n)
    xs = (LO + HI) / 2 + (HI - LO) / 2 * np.cos(np.pi * k[::-1] / (n - 1))
    grid = np.linspace(LO, HI, 200001)
    coeffs = None
    for _ in range(iters):
        # solve sum c_i x^i - E (-1)^k 2^x = 2^x  (relative-error equioscillation)
        a = np.zeros((n, n))
        for r, x in enumerate(xs):
            a[r, :degree + 1] = x ** np.arange(degree + 1)
            a[r, degree + 1] = (-1) ** r * 2.0 ** x
        sol = np.linalg.solve(a, 2.0 ** xs)
        coeffs = sol[:degree + 1]
        err = np.polyval(coeffs[::-1], grid) / 2.0 ** grid - 1.0
        # new reference: extrema of the error on each sign-alternating segment
        sign_changes = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate(([0], sign_changes + 1, [len(grid)]))
        ext = []
        for b0, b1 in zip(bounds[:-1], bounds[1:]):
            seg = np.abs(err[b0:b1])
            ext.append(b0 + int(np.argmax(seg)))
        if len(ext) != n:
            break
        xs = grid[ext]
    return coeffs


def float32_coeffs() -> np.ndarray:
    return remez().astype(np.float32)


def max_rel_error(coeffs: np.ndarray) -> float:
    f = np.linspace(LO, HI, 400001)
    p = np.polyval(coeffs.astype(np.float64)[::-1], f)
    return float(np.max(np.abs(p / 2.0 ** f - 1.0)))


if __name__ == "__main__":
    c = float32_coeffs()
    for i, v in enumerate(c):
        print(f"c{i} = {float(v)!r:>24}f  (0x{np.float32(v).view(np.uint32):08x})")
    print(f"max relative error on [-1/2, 1/2]: {max_rel_error(c):.3e}")
