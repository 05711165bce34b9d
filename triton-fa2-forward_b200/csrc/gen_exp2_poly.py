"""Fit the polynomial behind the kernel's FMA-pipe exp2 (exp2_poly.cuh).

Method (our own fit, not a copy of any library's constants):
  * Cody-Waite style split: x = n + f with n = round-to-nearest(x), f in [-1/2, 1/2];
    2^x = 2^n * 2^f, and 2^n is applied by adding n to the float's exponent field.
  * 2^f on [-1/2, 1/2] is approximated by a polynomial p(f) that minimises the maximum
    RELATIVE error, found with the Remez exchange algorithm (equioscillation of
    (p(f) - 2^f) / 2^f at degree + 2 reference points).
  * Coefficients are rounded to float32 and then re-checked with a float32 Horner
    evaluation on a dense grid, which is what the kernel executes.

Run:  python gen_exp2_poly.py      (prints the coefficient tables pasted into exp2_poly.cuh)
"""

import numpy as np


def remez_relative(deg, lo=-0.5, hi=0.5, iters=40):
    f = lambda x: np.exp2(x)
    n = deg + 2
    # Chebyshev extrema as the initial reference set
    k = np.arange(n)
    xs = 0.5 * (lo + hi) + 0.5 * (hi - lo) * -np.cos(np.pi * k / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    coef = None
    for _ in range(iters):
        # Solve sum_i c_i x^i - (-1)^j E f(x_j) = f(x_j)  (relative weighting 1/f)
        A = np.zeros((n, n))
        for j, x in enumerate(xs):
            A[j, : deg + 1] = x ** np.arange(deg + 1)
            A[j, deg + 1] = (-1) ** j * f(x)
        sol = np.linalg.solve(A, f(xs))
        coef = sol[: deg + 1]
        err = (np.polyval(coef[::-1], grid) - f(grid)) / f(grid)
        # new reference: extrema of the error between sign changes
        sgn = np.sign(err)
        idx = np.where(np.diff(sgn) != 0)[0]
        bounds = np.concatenate(([0], idx + 1, [len(grid)]))
        cand = []
        for a, b in zip(bounds[:-1], bounds[1:]):
            seg = np.abs(err[a:b])
            cand.append(a + int(np.argmax(seg)))
        cand = np.array(cand)
        if len(cand) > n:  # keep the n largest alternating extrema
            while len(cand) > n:
                mags = np.abs(err[cand])
                drop = np.argmin(mags)
                cand = np.delete(cand, drop)
        if len(cand) < n:
            break
        xs = grid[cand]
    return coef


def check_f32(coef):
    c = [np.float32(x) for x in coef]
    f = np.linspace(-0.5, 0.5, 400001, dtype=np.float32)
    p = np.full_like(f, c[-1])
    for ci in reversed(c[:-1]):
        p = (p * f + ci).astype(np.float32)
    ref = np.exp2(f.astype(np.float64))
    return float(np.max(np.abs(p.astype(np.float64) - ref) / ref))


if __name__ == "__main__":
    for deg in (3, 4, 5):
        coef = remez_relative(deg)
        rel = check_f32(coef)
        c32 = ", ".join(f"{np.float32(x).item():.9e}f" for x in coef)
        print(f"deg {deg}: max rel err (f32 Horner) {rel:.3e}")
        print(f"  c0..c{deg} = {{{c32}}}")
