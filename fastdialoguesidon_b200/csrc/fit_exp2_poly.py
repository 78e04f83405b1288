"""Fit the cubic used by the kernels' software 2^x (csrc/fds_ptx.cuh, exp2_poly).

Method: x = j + f with j = round(x) (round-to-nearest via the 1.5 * 2^23
shifter) and f in [-1/2, 1/2]; 2^x = 2^j * q(f) with q a degree-3 polynomial
minimising the maximum RELATIVE error |q(f) / 2^f - 1| on [-1/2, 1/2]
(Remez exchange on the weighted error). Prints the coefficients and the
achieved bound; the values are pasted into fds_ptx.cuh.
"""

import numpy as np


def remez_relative(deg: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 30):
    n = deg + 2
    # initial reference: Chebyshev extrema
    k = np.arange(n)
    x = (lo + hi) / 2 + (hi - lo) / 2 * np.cos(np.pi * k / (n - 1))[::-1]
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        f = np.exp2(x)
        # solve sum_i c_i x^i - f = (-1)^k E f  (relative error)
        a = np.zeros((n, n))
        for r in range(n):
            a[r, :deg + 1] = x[r] ** np.arange(deg + 1)
            a[r, deg + 1] = -((-1) ** r) * f[r]
        sol = np.linalg.solve(a, f)
        c, e = sol[:deg + 1], sol[deg + 1]
        err = (np.polyval(c[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        # new reference: extrema of err between sign changes
        idx = []
        sgn = np.sign(err)
        start = 0
        for i in range(1, len(grid) + 1):
            if i == len(grid) or sgn[i] != sgn[start]:
                seg = np.arange(start, i)
                idx.append(seg[np.argmax(np.abs(err[seg]))])
                start = i
        if len(idx) >= n:
            # keep the n largest alternating extrema
            idx = sorted(idx, key=lambda t: -abs(err[t]))[:n]
            x = np.sort(grid[idx])
    return c, float(np.max(np.abs(err)))


if __name__ == "__main__":
    c, e = remez_relative()
    c32 = c.astype(np.float32)
    g = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    q = ((c32[3] * g + c32[2]) * g + c32[1]) * g + c32[0]
    rel = np.max(np.abs(q.astype(np.float64) / np.exp2(g.astype(np.float64)) - 1))
    for i, v in enumerate(c32):
        print(f"c{i} = {float(v)!r}f  // {v.view(np.uint32):#010x}")
    print(f"minimax relative error {e:.3e}; fp32 Horner {rel:.3e}")
