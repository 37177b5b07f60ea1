"""Derive the polynomial the flash kernel uses for part of its exp2 evaluations.

Method: Cody-Waite style range reduction x = j + f with j = round(x) and
f in [-1/2, 1/2], so 2^x = 2^j * 2^f; 2^j is applied by adding j to the fp32
exponent field, and 2^f is approximated by a degree-4 polynomial whose
coefficients minimise the maximum RELATIVE error on [-1/2, 1/2] (Remez
exchange algorithm on the weighted error (p(f) - 2^f) / 2^f, with c0 pinned
so that p(0) = 1 exactly).  The printed coefficients are rounded to fp32 and
the error is re-measured in fp32 arithmetic with Horner's scheme, the order
the kernel evaluates it in.

Run: python animaxs_b200/csrc/gen_exp2_poly.py
"""

import numpy as np

DEG = 4
LO, HI = -0.5, 0.5


def remez(deg: int, iters: int = 60):
    # unknowns: c1..c_deg (c0 = 1) and the levelled error E; deg + 1 reference points
    n = deg + 1
    k = np.arange(n)
    xs = 0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * (n - 1 - k) / (n - 1))
    xs[np.isclose(xs, 0.0)] = 1e-3
    coef = None
    for _ in range(iters):
        a = np.zeros((n, n))
        rhs = np.zeros(n)
        for i, x in enumerate(xs):
            t = 2.0 ** x
            for p in range(1, deg + 1):
                a[i, p - 1] = x ** p / t
            a[i, deg] = (-1) ** i
            rhs[i] = 1.0 - 1.0 / t          # (1 + sum c_p x^p)/t - 1 = +-E
        sol = np.linalg.solve(a, rhs)
        coef = np.concatenate([[1.0], sol[:deg]])
        grid = np.linspace(LO, HI, 200001)
        err = np.polyval(coef[::-1], grid) / 2.0 ** grid - 1.0
        # new reference: the extrema of the error between sign changes, skipping f = 0
        idx = [0]
        for i in range(1, len(grid) - 1):
            if (err[i] - err[i - 1]) * (err[i + 1] - err[i]) <= 0 and abs(grid[i]) > 1e-4:
                idx.append(i)
        idx.append(len(grid) - 1)
        idx = sorted(idx, key=lambda i: -abs(err[i]))[:n]
        xs = np.sort(grid[idx])
    return coef


def horner_fp32(c, f):
    acc = np.float32(c[-1])
    for ci in c[-2::-1]:
        acc = np.float32(np.float32(acc * f) + np.float32(ci))
    return acc


def main():
    c = remez(DEG)
    c32 = [np.float32(v) for v in c]
    grid = np.linspace(LO, HI, 100001).astype(np.float32)
    approx = np.array([horner_fp32(c32, f) for f in grid[::10]], dtype=np.float64)
    exact = 2.0 ** grid[::10].astype(np.float64)
    rel = np.abs(approx / exact - 1.0).max()
    for i, v in enumerate(c32):
        print(f"c{i} = {float(v)!r:>24}  ({v.view(np.uint32):#010x})")
    print(f"max relative error (fp32 Horner, [-0.5, 0.5]): {rel:.3e}")


if __name__ == "__main__":
    main()
