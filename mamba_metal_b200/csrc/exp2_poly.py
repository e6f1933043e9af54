"""Derives the degree-5 polynomial of exp2_poly2 (mm_common.cuh): the minimax fit, in relative error, of
2^f on [-1/2, 1/2] by the Remez exchange algorithm, and checks the float32 Horner evaluation (one
rounding per fused multiply-add) on a dense grid. Prints the coefficients c0..c5 (as float32) and the
maximum relative error. Not used at run time.

    python mamba_metal_b200/csrc/exp2_poly.py
"""

import numpy as np


def remez(deg, a=-0.5, b=0.5, iters=30, grid_n=200001):
    k = np.arange(deg + 2)
    x = (a + b) / 2 + (b - a) / 2 * np.cos(np.pi * k[::-1] / (deg + 1))   # Chebyshev extrema
    grid = np.linspace(a, b, grid_n)
    for _ in range(iters):
        # p(x_i) - 2^x_i = (-1)^i E 2^x_i at the reference points (equioscillating relative error)
        m = np.zeros((deg + 2, deg + 2))
        for i in range(deg + 2):
            m[i, :deg + 1] = x[i] ** np.arange(deg + 1)
            m[i, deg + 1] = -((-1) ** i) * 2 ** x[i]
        sol = np.linalg.solve(m, 2 ** x)
        c = sol[:deg + 1]
        r = np.polyval(c[::-1], grid) / 2 ** grid - 1
        segs = np.split(np.arange(grid_n), np.nonzero(np.diff(np.sign(r)))[0] + 1)
        ext = sorted(sorted((s[np.argmax(np.abs(r[s]))] for s in segs), key=lambda i: -abs(r[i]))[:deg + 2])
        x = grid[ext]
    return c


def main():
    c32 = remez(5).astype(np.float32)
    f = np.linspace(-0.5, 0.5, 2000001).astype(np.float32)
    p = np.full_like(f, c32[5])
    for k in range(4, -1, -1):
        p = (p.astype(np.float64) * f + np.float64(c32[k])).astype(np.float32)   # one rounding per FMA
    rel = np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1)
    print("c0..c5 =", ", ".join(f"{v:.8g}" for v in c32))
    print(f"max relative error of the float32 evaluation: {rel.max():.3g} ({rel.max() / 2 ** -23:.2f} ulp)")


if __name__ == "__main__":
    main()
