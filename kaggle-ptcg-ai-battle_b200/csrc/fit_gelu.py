"""Coefficients of the tensor-core epilogue's GELU (common.cuh, gelu2).

The epilogue writes Phi(x) = 1/2 + sign(x) (1/2 - q(x)) with the normal
tail q(x) = erfc(|x| / sqrt 2) / 2 = pdf(x) P(|x|), where pdf is the normal
density (one ex2 per element, shared with GELU' = Phi + x pdf) and

    P(u) = sqrt(pi / 2) erfcx(u / sqrt 2)

is smooth and bounded on u in [0, 4 sqrt 2].  P is fitted by a polynomial
whose error is weighted by pdf(u) (the error that reaches Phi), driven to
equal ripple by Lawson's iteratively reweighted least squares.  The
coefficients are printed negated (the epilogue evaluates 1/2 - q as one
fma) in float32, and the float32 Horner evaluation is checked here.

    python fit_gelu.py [degree]
"""
import sys

import numpy as np
from scipy.special import erfcx

UMAX = 4.0 * np.sqrt(2.0)


def fit(deg, n=200001, iters=80):
    u = np.linspace(0.0, UMAX, n)
    target = np.sqrt(np.pi / 2) * erfcx(u / np.sqrt(2.0))
    w = np.exp(-0.5 * u * u) / np.sqrt(2 * np.pi)
    V = np.vander(u, deg + 1, increasing=True)
    lw = np.ones_like(u)
    for _ in range(iters):
        sw = np.sqrt(lw) * w
        c, *_ = np.linalg.lstsq(V * sw[:, None], target * sw, rcond=None)
        e = np.abs(V @ c - target) * w
        lw *= e / e.max() + 1e-15
        lw /= lw.mean()
    c32 = (-c).astype(np.float32)
    p = np.full(n, c32[-1], np.float32)
    uf = u.astype(np.float32)
    for k in range(deg - 1, -1, -1):
        p = p * uf + c32[k]
    err = np.abs(-p.astype(np.float64) - target) * w   # |q error| = |Phi error|
    return c32, err.max()


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 7
    c, e = fit(deg)
    print(f"degree {deg}: max |Phi error| {e:.3e} (float32 Horner)")
    for k in range(deg, -1, -1):
        print(f"  c{k} = {c[k]:.9e}f")
