"""Coefficients of the polynomials p(f) ~ 2^f on [-0.5, 0.5] used by the
prefill kernels' FMA-pipe exponentials (prefill.cu, f2_exp2_poly): degree 3
for the softmax, degree 4 for the softcap's tanh.

Method: weighted least squares (relative error) at 2000 Chebyshev nodes,
rounded to float32; the script prints the coefficients and the maximum
relative error of the float32 Horner evaluation: degree 3 7.7e-5 (below the
4.9e-4 rounding of the fp16 P operand), degree 4 2.7e-6 (tanh error at most
1.4e-6, 7e-5 in a score capped at 50). Run: python aspida_b200/csrc/exp2_poly_fit.py
"""
import numpy as np


def fit(deg=3, n=2000):
    k = np.arange(n)
    x = 0.5 * np.cos((2 * k + 1) * np.pi / (2 * n))
    w = 1.0 / np.exp2(x)
    c, *_ = np.linalg.lstsq(np.vander(x, deg + 1, increasing=True) * w[:, None], np.exp2(x) * w,
                            rcond=None)
    return c.astype(np.float32)


def max_rel_err(c):
    t = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.full_like(t, c[-1])
    for ci in c[-2::-1]:
        p = (p * t + ci).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) / np.exp2(t.astype(np.float64)) - 1)))


if __name__ == "__main__":
    for deg in (3, 4):
        c = fit(deg)
        print(f"degree {deg}: coefficients c0..c{deg}:", ", ".join(f"{float(v):.9g}f" for v in c))
        print("  max relative error:", max_rel_err(c))
