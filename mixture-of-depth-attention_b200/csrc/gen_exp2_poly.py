"""Coefficients of the software base-2 exponential used by the tcgen05 kernel.

Method (published): Cody & Waite range reduction (W. J. Cody, W. Waite,
"Software Manual for the Elementary Functions", 1980): x = n + f with
n = round(x), f in [-1/2, 1/2], 2^x = 2^n * 2^f; 2^n is applied by adding n to
the IEEE-754 exponent field. 2^f is a degree-3 polynomial whose coefficients
minimise the maximum RELATIVE error on [-1/2, 1/2], found with the Remez
exchange algorithm (E. Ya. Remez, 1934).

    python mixture-of-depth-attention_b200/csrc/gen_exp2_poly.py

prints the coefficients (rounded to fp32) and the resulting error bound. The
kernel rounds P to bf16/f16 (relative step 2^-8 / 2^-11), so a relative error
near 1e-4 is far below the rounding the MMA sees.
"""

import numpy as np

DEG = 3
LO, HI = -0.5, 0.5


def remez_relative(deg=DEG, iters=40):
    f = lambda x: np.exp2(x)
    # initial reference: Chebyshev extrema
    k = np.arange(deg + 2)
    xs = 0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * k / (deg + 1))[::-1]
    grid = np.linspace(LO, HI, 200001)
    for _ in range(iters):
        # solve p(x_i) - f(x_i) = (-1)^i E f(x_i)  (relative equioscillation)
        A = np.zeros((deg + 2, deg + 2))
        for i, x in enumerate(xs):
            A[i, :deg + 1] = x ** np.arange(deg + 1)
            A[i, deg + 1] = -((-1) ** i) * f(x)
        sol = np.linalg.solve(A, f(xs))
        c = sol[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        # new reference: extrema of the error between sign changes
        idx = [0]
        sign = np.sign(err)
        for i in range(1, len(grid)):
            if sign[i] != sign[idx[-1]]:
                idx.append(i)
            elif abs(err[i]) > abs(err[idx[-1]]):
                idx[-1] = i
        if len(idx) >= deg + 2:
            best = max(range(len(idx) - deg - 1),
                       key=lambda s: min(abs(err[j]) for j in idx[s:s + deg + 2]))
            xs = grid[idx[best:best + deg + 2]]
    return c, float(np.max(np.abs(err)))


def emulate(x, c):
    """fp32 model of the kernel's sequence: clamp, round via 1.5*2^23, Horner, exponent add."""
    x = np.maximum(np.float32(x), np.float32(-125.0)).astype(np.float32)
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    fr = (x - n).astype(np.float32)
    c32 = [np.float32(v) for v in c]
    p = (c32[3] * fr + c32[2]).astype(np.float32)
    p = (p * fr + c32[1]).astype(np.float32)
    p = (p * fr + c32[0]).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.view(np.float32)


if __name__ == "__main__":
    c, e = remez_relative()
    c32 = [float(np.float32(v)) for v in c]
    xs = np.linspace(-125, 8, 2_000_001).astype(np.float32)
    rel = np.abs(emulate(xs, c32).astype(np.float64) / np.exp2(xs.astype(np.float64)) - 1)
    print("coefficients c0..c3 (fp32):", ", ".join(f"{v:.9e}f" for v in c32))
    print(f"minimax relative error on [-1/2,1/2]: {e:.3e}; fp32 pipeline on [-125, 8]: {rel.max():.3e}")
