"""Fit the polynomial used by fe::exp2_poly (fe_ptx.cuh).

Method: Cody-Waite style range reduction x = n + f with n = rint(x),
f in [-1/2, 1/2], then 2^f by a polynomial whose coefficients minimise the
maximum relative error on [-1/2, 1/2] (Remez exchange on the relative error,
starting from Chebyshev extrema).  2^n is applied by adding n to the exponent
field.  Run to regenerate the constants:

    python flash-evict-prefill_b200/csrc/fit_exp2.py [degree]
"""
import sys

import numpy as np


def remez_relative(degree, lo=-0.5, hi=0.5, iters=30):
    f = lambda x: np.exp2(x)  # noqa: E731
    n = degree + 2
    k = np.arange(n)
    x = (lo + hi) / 2 + (hi - lo) / 2 * np.cos(np.pi * k / (n - 1))[::-1]
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        # Solve sum_j c_j x_i^j - f(x_i) = (-1)^i E f(x_i)
        a = np.zeros((n, n))
        for i in range(n):
            a[i, :degree + 1] = x[i] ** np.arange(degree + 1)
            a[i, degree + 1] = -((-1) ** i) * f(x[i])
        sol = np.linalg.solve(a, f(x))
        c = sol[:degree + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        # new reference: extrema of the error between sign changes
        sign = np.sign(err)
        idx = [0]
        for i in range(1, len(grid)):
            if sign[i] != sign[idx[-1]]:
                idx.append(i)
            elif abs(err[i]) > abs(err[idx[-1]]):
                idx[-1] = i
        if len(idx) < n:
            break
        # keep the n largest alternating extrema
        while len(idx) > n:
            if abs(err[idx[0]]) < abs(err[idx[-1]]):
                idx.pop(0)
            else:
                idx.pop()
        x = grid[idx]
    return c, np.abs(err).max()


def fp32_eval_error(c):
    xs = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    p = np.float32(c[-1])
    for cc in c[-2::-1]:
        p = (p * xs + np.float32(cc)).astype(np.float32)
    return np.abs((p.astype(np.float64) - np.exp2(xs.astype(np.float64))) / np.exp2(xs.astype(np.float64))).max()


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 5
    c, e = remez_relative(deg)
    print(f"degree {deg}: max relative error {e:.3e} (exact arithmetic), {fp32_eval_error(c):.3e} (fp32 Horner)")
    for i, cc in enumerate(c):
        print(f"  c{i} = {np.float32(cc).item()!r}f  // {cc!r}")
