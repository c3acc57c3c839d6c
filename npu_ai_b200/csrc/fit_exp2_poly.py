"""Fits the polynomial behind exp2_poly3() in sm100_ptx.cuh.

2^f on f in [-1/2, 1/2] by p(f) = 1 + c1 f + c2 f^2 + c3 f^3 (p(0) = 1 exactly, so 2^n comes out exact for integer
inputs), chosen to minimise the maximum RELATIVE error |p(f) / 2^f - 1| over a dense grid: a linear program in
(c1, c2, c3, e) with |p(f) - 2^f| <= e * 2^f at every grid point (Chebyshev / minimax fit by linear programming).
The coefficients are rounded to f32 and the achieved error is re-measured in f32 arithmetic.

Run: python npu_ai_b200/csrc/fit_exp2_poly.py
"""
import numpy as np
from scipy.optimize import linprog


def fit(n_grid: int = 4001):
    f = np.linspace(-0.5, 0.5, n_grid)
    y = np.exp2(f)
    # variables: c1, c2, c3, e ; minimise e
    A = np.stack([f, f ** 2, f ** 3], axis=1)
    # p - y <= e y  ->  A c - e y <= y - 1 ;  y - p <= e y  ->  -A c - e y <= 1 - y
    A_ub = np.vstack([np.hstack([A, -y[:, None]]), np.hstack([-A, -y[:, None]])])
    b_ub = np.concatenate([y - 1.0, 1.0 - y])
    res = linprog(c=[0, 0, 0, 1], A_ub=A_ub, b_ub=b_ub, bounds=[(None, None)] * 3 + [(0, None)], method="highs")
    assert res.success, res.message
    return np.float32(res.x[:3]), float(res.x[3])


def poly_f32(x, c):
    """The kernel's evaluation order, in f32: clamp, round-to-nearest split, Horner, exponent add."""
    x = np.maximum(np.float32(x), np.float32(-125.0)).astype(np.float32)
    t = (x + np.float32(12582912.0)).astype(np.float32)
    n = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = np.float32(c[2]) * f + np.float32(c[1])
    p = (p * f + np.float32(c[0])).astype(np.float32)
    p = (p * f + np.float32(1.0)).astype(np.float32)
    bits = (t.view(np.int32).astype(np.int64) << 23).astype(np.int64) & 0xFFFFFFFF
    out = ((p.view(np.int32).astype(np.int64) + bits) & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return out


if __name__ == "__main__":
    c, e = fit()
    xs = np.linspace(-60.0, 8.0, 2_000_001).astype(np.float32)
    rel = np.abs(poly_f32(xs, c).astype(np.float64) / np.exp2(xs.astype(np.float64)) - 1.0).max()
    print("c1, c2, c3 =", ", ".join(f"{v:.9e}f" for v in c))
    print(f"LP minimax relative error {e:.3e}; measured in f32 on [-60, 8]: {rel:.3e}")
