"""Derives the polynomial of the GELU epilogue (csrc/gelu.cuh).

GELU(x) = x * Phi(x), Phi(x) = 1 - erfc(x/sqrt2)/2 for x >= 0 and
erfc(|x|/sqrt2)/2 for x < 0.  With u = |x|,

    erfc(u/sqrt2) = erfcx(u/sqrt2) * exp(-u^2/2)
                  = 2^( Q(u) - u^2 * log2(e)/2 ),   Q(u) = log2(erfcx(u/sqrt2)),

where erfcx(z) = exp(z^2) erfc(z) is smooth and slowly varying.  Q is
approximated on [0, U0] by a Chebyshev least-squares fit of degree DEG,
converted to monomial coefficients for Horner evaluation in fp32.  Beyond
U0 = 4.5, erfc(u/sqrt2) < 6.8e-6 and u is clamped inside Q only: the exact
-u^2 term keeps the decay, and Q(U0) >= Q(u) overestimates erfc by a factor
below u/U0, an absolute GELU error below 1e-6 (2e-9 at u = 6).

Run:  python csrc/gelu_fit.py   (prints the coefficient table and the
fp32-simulated error of GELU against the exact function).
"""
import numpy as np
from numpy.polynomial import chebyshev as C
from numpy.polynomial import polynomial as P
from scipy.special import erfc, erfcx

U0 = 4.5
DEG = 6


def fit():
    u = np.linspace(0.0, U0, 400001)
    q = np.log2(erfcx(u / np.sqrt(2.0)))
    c = C.chebfit(u * (2.0 / U0) - 1.0, q, DEG)
    mono_t = C.cheb2poly(c)
    pu = np.zeros(1)
    for k, ck in enumerate(mono_t):
        pu = P.polyadd(pu, ck * P.polypow([-1.0, 2.0 / U0], k))
    return pu.astype(np.float32)


def gelu_fp32(x, coef):
    """fp32 simulation of the kernel's evaluation order (gelu.cuh): Horner
    with the constant term lowered by 1 (the factor 1/2 of erfc/2), then
    GELU(x) = max(x, 0) - |x| * 2^q."""
    x = x.astype(np.float32)
    u = np.abs(x)
    uc = np.minimum(u, np.float32(U0))
    c = coef.copy()
    c[0] = np.float32(c[0] - np.float32(1.0))
    acc = np.full_like(x, c[-1])
    for ck in c[-2::-1]:
        acc = (acc * uc + ck).astype(np.float32)
    q = (x * x * np.float32(-0.5 * np.log2(np.e)) + acc).astype(np.float32)
    h = np.exp2(q).astype(np.float32)
    return (np.maximum(x, np.float32(0.0)) - u * h).astype(np.float32)


if __name__ == "__main__":
    coef = fit()
    x = np.linspace(-12, 12, 2_000_001)
    exact = x * 0.5 * erfc(-x / np.sqrt(2.0))  # no cancellation for x << 0
    g = gelu_fp32(x, coef).astype(np.float64)
    abs_err = np.abs(g - exact)
    rel = abs_err / np.maximum(np.abs(exact), 1e-30)
    print("coefficients (u^0 .. u^%d):" % DEG)
    for k, ck in enumerate(coef):
        print(f"  {float(ck)!r}f,  // u^{k}")
    print(f"max abs err {abs_err.max():.3e}; max rel err {rel.max():.3e} "
          f"(on [-U0, U0]: {rel[np.abs(x) <= U0].max():.3e})")
