"""Derives the polynomial of the GELU epilogue (csrc/gelu.cuh).

GELU(x) = x * Phi(x), Phi(x) = 1 - erfc(x/sqrt2)/2 for x >= 0 and
erfc(|x|/sqrt2)/2 for x < 0.  With u = |x| and h(u) = erfc(u/sqrt2)/2,

    GELU(x) = max(x, 0) - u * h(u),   h(u) = 2^P(u),

where P(u) = log2(erfc(u/sqrt2)/2) = log2(erfcx(u/sqrt2)) - u^2 log2(e)/2 - 1
is smooth (the -u^2 decay is exactly a polynomial term).  P is approximated
on [0, U0] by a Chebyshev least-squares fit of degree DEG, converted to
monomial coefficients for Horner evaluation in fp32.  The kernel does not
clamp u: past U0 = 6 the polynomial keeps falling (P(6) = -29.9 is its
largest value there), so h stays below h(6) = 9.9e-10 and goes to 0, and
GELU(x) is within |x| * 9.9e-10 of max(x, 0).

Run:  python csrc/gelu_fit.py   (prints the coefficient table and the
fp32-simulated error of GELU against the exact function).
"""
import numpy as np
from numpy.polynomial import chebyshev as C
from numpy.polynomial import polynomial as P
from scipy.special import erfc

U0 = 6.0
DEG = 7


def fit():
    u = np.linspace(0.0, U0, 400001)
    p = np.log2(erfc(u / np.sqrt(2.0)) / 2.0)
    c = C.chebfit(u * (2.0 / U0) - 1.0, p, DEG)
    mono_t = C.cheb2poly(c)
    pu = np.zeros(1)
    for k, ck in enumerate(mono_t):
        pu = P.polyadd(pu, ck * P.polypow([-1.0, 2.0 / U0], k))
    return pu.astype(np.float32)


def gelu_fp32(x, coef):
    """fp32 simulation of the kernel's evaluation order (gelu.cuh): Horner
    on |x|, then GELU(x) = max(x, 0) - |x| * 2^P."""
    x = x.astype(np.float32)
    u = np.abs(x)
    uc = u  # no clamp (see the module docstring)
    acc = np.full_like(x, coef[-1])
    for ck in coef[-2::-1]:
        acc = (acc * uc + ck).astype(np.float32)
    h = np.exp2(acc).astype(np.float32)
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
    print(f"max abs err {abs_err.max():.3e}; max rel err on [-4.5, 4.5] "
          f"{rel[np.abs(x) <= 4.5].max():.3e}")
