#!/usr/bin/env python3
"""Coefficients of the polynomial exp2 used by the attention softmax.

2^x = 2^j * 2^f with j = rint(x) and f = x - j in [-0.5, 0.5]; 2^f is a
degree-4 polynomial fitted here by the Remez exchange algorithm on the
relative error over [-0.5, 0.5] (minimax), then rounded to fp32.  Running this
script prints the fp32 coefficients (lowest degree first) exactly as
`exp2_poly.cuh` holds them, and the maximum relative error of the exact and of
the fp32-rounded polynomial.
"""
import numpy as np

DEG = 4  # relative error 2.6e-6: far below the fp16 rounding (2^-11) of the P it feeds
LO, HI = -0.5, 0.5


def remez(deg=DEG, lo=LO, hi=HI, iters=30, n_grid=200001):
    n = deg + 2
    k = np.arange(n)
    xs = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * k[::-1] / (n - 1))
    grid = np.linspace(lo, hi, n_grid)
    f = np.exp2
    c = None
    for _ in range(iters):
        a = np.zeros((n, n))
        for i, x in enumerate(xs):
            a[i, :deg + 1] = x ** np.arange(deg + 1)
            a[i, deg + 1] = (-1) ** i * f(x)
        c = np.linalg.solve(a, f(xs))[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        sgn = np.sign(err)
        idx, start = [], 0
        for i in range(1, len(grid)):
            if sgn[i] != sgn[i - 1]:
                idx.append(start + int(np.argmax(np.abs(err[start:i]))))
                start = i
        idx.append(start + int(np.argmax(np.abs(err[start:]))))
        if len(idx) > n:
            idx = sorted(sorted(idx, key=lambda j: -abs(err[j]))[:n])
        if len(idx) == n:
            xs = grid[idx]
    return c


def coefficients_f32():
    return remez().astype(np.float32)


def max_rel_error(c, n_grid=200001):
    g = np.linspace(LO, HI, n_grid)
    return float(np.max(np.abs(np.polyval(np.asarray(c, np.float64)[::-1], g) / np.exp2(g) - 1.0)))


if __name__ == "__main__":
    c = remez()
    c32 = c.astype(np.float32)
    print("max relative error, exact coefficients:", max_rel_error(c))
    print("max relative error, fp32 coefficients: ", max_rel_error(c32))
    for i, v in enumerate(c32):
        print(f"c{i} = {float(v)!r:>24}  ({hex(int(np.float32(v).view(np.uint32)))})")
