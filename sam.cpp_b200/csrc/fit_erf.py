"""Fit of erf used by the GEMM epilogue's erf-GELU (gemm.cu, gelu_erf).

erf(z) on z in [0, 4] is fitted by a degree-17 Chebyshev least-squares fit
(401k nodes, reference values from Python's math.erf) and converted to the
power basis in u = (z - 2) / 2 in [-1, 1], evaluated by f32 Horner.  Max
absolute error over [0, 4] with f32 arithmetic: 2.9e-7 (erf(4) = 1 - 1.5e-8,
so z > 4 is clamped to erf = 1).  Run this file to print the coefficients.
"""
from math import erf

import numpy as np


def fit(degree=17):
    z = np.linspace(0.0, 4.0, 400001)
    values = np.array([erf(t) for t in z])
    cheb = np.polynomial.chebyshev.Chebyshev.fit(z, values, degree, domain=[0, 4])
    power = np.polynomial.chebyshev.cheb2poly(cheb.coef).astype(np.float32)
    u = ((z.astype(np.float32) - np.float32(2)) * np.float32(0.5)).astype(np.float32)
    acc = np.full_like(u, power[-1])
    for c in power[-2::-1]:
        acc = (acc * u + c).astype(np.float32)
    return power, float(np.abs(acc.astype(np.float64) - values).max())


if __name__ == "__main__":
    coefficients, error = fit()
    print("max abs error", error)
    print(", ".join(f"{c!r}f" for c in coefficients.tolist()))
