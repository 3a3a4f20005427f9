"""Derives the polynomial the GEMM epilogues' exact-erf GELU uses (gemm.cuh, GeluK / gelu_pair).

GELU(x) = x * Phi(x) (F.gelu with approximate="none"). With a = |x| and q(a) = Phi(-a) = erfc(a / sqrt(2)) / 2,
GELU(x) = relu(x) - a * q(a) for either sign of x, with no cancellation. log2 q(a) is smooth on [0, 10]
(from -1 at a = 0 to about -76.8 at a = 10, dominated by -a^2 / (2 ln 2)), so a polynomial P in
u = a / 5 - 1 in [-1, 1] fits it closely, and q = 2^P(u) takes one 2^x on the special-function unit per value
and no division. Past a = 10, a is clamped: q(10) = 7.6e-24, so GELU is x (x > 10) or below 1e-21 in magnitude
(x < -10).

The fit: least squares in the Chebyshev basis on NODES Chebyshev nodes of [-1, 1] (close to the minimax
polynomial), converted to monomial coefficients in u for Horner's rule. log2 q is evaluated with
scipy.special.log_ndtr (accurate in the far tail, where 1 - Phi cancels). Run it to print the coefficients and
the relative error of q = 2^P over [0, 10] in float32 arithmetic (Horner with one rounding per step):

    python mayfly_chess_b200/csrc/gelu_poly.py
"""
import numpy as np
from scipy.special import log_ndtr

DEGREE = 8
NODES = 4000
A_MAX = 10.0


def coefficients(degree=DEGREE, nodes=NODES):
    """Monomial coefficients c[0..degree] of P(u) ~ log2 Phi(-5 (u + 1)), lowest power first."""
    k = np.arange(nodes)
    u = np.cos(np.pi * (k + 0.5) / nodes)
    a = (A_MAX / 2) * (u + 1)
    cheb = np.polynomial.chebyshev.chebfit(u, log_ndtr(-a) / np.log(2), degree)
    return np.polynomial.chebyshev.cheb2poly(cheb)


def float32_error(c, samples=400001):
    """max relative error of 2^P(u) against q(a) over a in [0, A_MAX], P evaluated in float32."""
    a = np.linspace(0, A_MAX, samples).astype(np.float32)
    u = (a * np.float32(2 / A_MAX) + np.float32(-1)).astype(np.float32)
    c32 = c.astype(np.float32)
    p = np.full_like(u, c32[-1])
    for ci in c32[-2::-1]:
        p = (p * u + ci).astype(np.float32)
    exact = log_ndtr(-a.astype(np.float64)) / np.log(2)
    return float(np.abs(np.exp2(p.astype(np.float64) - exact) - 1).max())


if __name__ == "__main__":
    c = coefficients()
    for i, v in enumerate(c):
        print(f"c{i} = {np.float32(v)!r:>16}  ({v:.12e})")
    print(f"max relative error of q in float32 over [0, {A_MAX:g}]: {float32_error(c):.3e}")
