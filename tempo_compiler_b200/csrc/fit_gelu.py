"""Derives the coefficients of `gelu_erf` (common.cuh) and checks its float32 evaluation.

GELU(x) = x Phi(x) with Phi(x) = 1 - c for x >= 0 and c for x < 0, where c = erfc(|x| / sqrt 2) / 2. With
z = |x| / sqrt 2 and t = 1 / (1 + z / 2) (t in (0, 1] for z >= 0), c is written as

    c = t * 2^(P(t) - z^2 log2(e)),        P(t) ~ log2(erfcx(z) / (2 t)),

erfcx(z) = e^(z^2) erfc(z) being smooth and bounded on [0, inf). This is the classical substitution behind the
Chebyshev-fitted erfc of Press et al., Numerical Recipes (2nd ed., section 6.2); the polynomial here is this project's
own fit: degree 8 in t over z in [0, 9.5] (below 0.5 erfc(9.5) ~ 2e-41 the float32 result is flushed to zero
anyway), near-minimax in the absolute error of P (= relative error of c / ln 2) by Lawson's iteratively reweighted
least squares on 4000 Chebyshev nodes, against scipy.special.erfcx.

Run as a script it prints the coefficients (lowest order first) and the float32 evaluation's worst relative error
over every finite BF16 value with |x| <= 14. The CPU test suite imports `fit()` and `evaluate_float32()` to check that
the constants compiled into the kernels are these and that the evaluation stays within its bound.
"""
from __future__ import annotations

import math

import numpy as np

DEGREE = 8
Z_MAX = 9.5


def _lawson(x: np.ndarray, y: np.ndarray, degree: int, relative: bool, iterations: int) -> np.ndarray:
    """Near-minimax polynomial through Lawson's iteratively reweighted least squares (absolute or relative error)."""
    vander = np.vander(x, degree + 1, increasing=True)
    scale = 1.0 / y if relative else np.ones_like(y)
    weights = np.ones_like(x)
    coeffs = np.zeros(degree + 1)
    for _ in range(iterations):
        root = np.sqrt(weights) * scale
        coeffs, *_ = np.linalg.lstsq(vander * root[:, None], y * root, rcond=None)
        weights = weights * (np.abs(vander @ coeffs - y) * scale + 1e-30)
        weights /= weights.sum()
    return coeffs


def _target(t: np.ndarray) -> np.ndarray:
    from scipy.special import erfcx
    z = 2.0 * (1.0 / t - 1.0)
    return np.log2(0.5 * erfcx(z) / t)


def fit(degree: int = DEGREE, nodes: int = 4000, iterations: int = 60) -> np.ndarray:
    """Coefficients of the GELU tail's P, lowest order first (float64)."""
    t_min = 1.0 / (1.0 + 0.5 * Z_MAX)
    k = np.arange(nodes)
    t = (t_min + 1.0) / 2 + (1.0 - t_min) / 2 * np.cos(np.pi * (k + 0.5) / nodes)
    return _lawson(t, _target(t), degree, relative=False, iterations=iterations)


def evaluate_float32(x: np.ndarray, coeffs: np.ndarray) -> np.ndarray:
    """The kernels' evaluation order in float32 (the reciprocal and 2^e taken as correctly rounded; the GPU's
    approximate instructions add about one unit in the last place to each)."""
    f = np.float32
    c = np.asarray(coeffs, dtype=np.float32)
    x = np.asarray(x, dtype=np.float32)
    t = (f(1) / (np.abs(x) * f(0.5 / math.sqrt(2.0)) + f(1))).astype(np.float32)
    p = np.full_like(x, c[-1])
    for j in range(len(c) - 2, -1, -1):
        p = (p * t + c[j]).astype(np.float32)
    e = (x * (x * f(-0.5 / math.log(2.0))) + p).astype(np.float32)
    tail = (t * np.exp2(e)).astype(np.float32)
    return (x * np.where(x < 0, tail, f(1) - tail)).astype(np.float32)


def exact(x: np.ndarray) -> np.ndarray:
    from scipy.special import erfc
    xd = np.asarray(x, dtype=np.float64)
    return 0.5 * xd * erfc(-xd / math.sqrt(2.0))


def bf16_inputs(limit: float = 14.0) -> np.ndarray:
    bits = (np.arange(1 << 16, dtype=np.uint32) << 16).view(np.float32)
    return bits[np.isfinite(bits) & (np.abs(bits) <= limit) & (np.abs(bits) >= 1e-30)]


if __name__ == "__main__":
    coeffs = fit()
    print("GELU coefficients:", ", ".join(f"{float(np.float32(c))!r}f" for c in coeffs))
    x = bf16_inputs()
    ref = exact(x)
    keep = np.abs(ref) > 1e-37
    rel = np.abs(evaluate_float32(x, coeffs) - ref)[keep] / np.abs(ref[keep])
    print(f"float32 evaluation: worst relative error {rel.max():.3g} over {keep.sum()} BF16 inputs")
