"""Fit of the polynomial behind ex2x2_fma (common.cuh): 2^r on [-1/2, 1/2], degree 5,
minimising the maximum RELATIVE error by the Remez exchange algorithm, in float64.

    python swiftx_b200/csrc/fit_exp2_poly.py

prints the coefficients c0..c5 (rounded to float32, as common.cuh holds them), the
minimax error of the float64 fit, and the error of the whole float32 pipeline (round x to
an integer j with the 1.5 * 2^23 constant, r = x - j, Horner with fused multiply-adds,
2^j added to the exponent field) over [-125, 4].
"""
import numpy as np

DEG, LO, HI = 5, -0.5, 0.5


def remez(deg=DEG, iters=40):
    f = np.exp2
    grid = np.linspace(LO, HI, 200001)
    # start from the Chebyshev extrema
    xs = np.sort(0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * np.arange(deg + 2) / (deg + 1)))
    for _ in range(iters):
        # p(x_i) - f(x_i) = (-1)^i E f(x_i): the relative error equioscillates with size E
        A = np.array([[x ** k for k in range(deg + 1)] + [(-1) ** i * f(x)] for i, x in enumerate(xs)])
        sol = np.linalg.solve(A, f(xs))
        c = sol[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        # next reference: one extremum of the error per sign run, deg + 2 of them
        runs, start = [], 0
        s = np.sign(err)
        for i in range(1, len(grid) + 1):
            if i == len(grid) or s[i] != s[start]:
                seg = slice(start, i)
                runs.append(start + int(np.argmax(np.abs(err[seg]))))
                start = i
        if len(runs) < deg + 2:
            break
        while len(runs) > deg + 2:                     # drop the smaller end extremum
            runs.pop(0 if abs(err[runs[0]]) < abs(err[runs[-1]]) else -1)
        xs = grid[runs]
    return c, np.abs(err).max()


def pipeline_error(c32):
    x = np.linspace(-125, 4, 2_000_001).astype(np.float32)
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    r = (x - j).astype(np.float32)
    p = np.full_like(r, c32[DEG])
    for ci in c32[DEG - 1::-1]:
        p = (p.astype(np.float64) * r + np.float64(ci)).astype(np.float32)    # one rounding per fma
    y = (p.view(np.int32) + (t.view(np.int32) << 23)).view(np.float32)
    ref = np.exp2(x.astype(np.float64))
    return np.max(np.abs(y.astype(np.float64) - ref) / ref)


if __name__ == "__main__":
    c, e = remez()
    c32 = c.astype(np.float32)
    print("c0..c5 (float32):", ", ".join(repr(float(v)) for v in c32))
    print(f"minimax relative error (float64 fit): {e:.3e}")
    print(f"float32 pipeline relative error over [-125, 4]: {pipeline_error(c32):.3e}")
