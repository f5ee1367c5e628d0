"""Lloyd-Max codebooks for rotated unit-vector coordinates.

Host-side, one-time table generation.  The iteration is the one the reference
uses (aditya25058/Bhaskera_col src/bhaskera/inference/lloyd_max.py:44-100) so
that the fp32 centroids and boundaries come out bit-identical: they decide
every stored code, and the kernels compare against these exact fp32 values.

  * density: N(0, 1/d) (or the exact Beta-type marginal of a uniformly random
    unit vector when use_exact_pdf=True)
  * start: 2^b centroids uniform on [-4s, 4s], s = 1/sqrt(d)
  * step: cells bounded by centroid midpoints, outer edges at +-8s; each
    centroid moves to its cell's conditional mean, integrals by adaptive
    quadrature (scipy.integrate.quad, limit=200)
  * stop: largest centroid move < tol (1e-12) or 300 steps
  * boundaries: midpoints of the final centroids
"""
from __future__ import annotations

import logging
import math
from typing import Callable, Dict, Tuple

import torch

logger = logging.getLogger(__name__)


def _normal_density(var: float) -> Callable[[float], float]:
    # evaluated exactly as written (no hoisted constant) so every quadrature
    # node sees the same rounding as the reference's density
    def f(x):
        x = float(x)
        return math.exp(-x * x / (2.0 * var)) / math.sqrt(2.0 * math.pi * var)
    return f


def _sphere_marginal(d: int) -> Callable[[float], float]:
    c = math.gamma(d / 2) / (math.sqrt(math.pi) * math.gamma((d - 1) / 2))

    def f(x):
        x = float(x)
        return 0.0 if abs(x) >= 1.0 else c * (1.0 - x * x) ** ((d - 3) / 2)
    return f


def _quad(fn, a: float, b: float) -> float:
    try:
        from scipy.integrate import quad
    except ImportError:  # midpoint rule, as the reference does without scipy
        n = 1000
        dx = (b - a) / n
        return sum(fn(a + (i + 0.5) * dx) * dx for i in range(n))
    return quad(fn, a, b, limit=200)[0]


def solve_lloyd_max(d: int, bits: int, use_exact_pdf: bool = False, max_iter: int = 300,
                    tol: float = 1e-12) -> Tuple[torch.Tensor, torch.Tensor]:
    """Return (centroids [2^bits], boundaries [2^bits - 1]) as fp32 tensors."""
    levels = 1 << bits
    var = 1.0 / d
    sd = math.sqrt(var)
    lo, hi = -4.0 * sd, 4.0 * sd
    dens = _sphere_marginal(d) if use_exact_pdf else _normal_density(var)

    def first_moment(x):
        return x * dens(x)

    cents = [lo + (hi - lo) * (k + 0.5) / levels for k in range(levels)]
    for _ in range(max_iter):
        cuts = [lo * 2] + [(cents[k] + cents[k + 1]) / 2.0 for k in range(levels - 1)] + [hi * 2]
        moved = 0.0
        nxt = []
        for k in range(levels):
            mass = _quad(dens, cuts[k], cuts[k + 1])
            mean = _quad(first_moment, cuts[k], cuts[k + 1]) / mass if mass > 1e-15 else cents[k]
            moved = max(moved, abs(mean - cents[k]))
            nxt.append(mean)
        cents = nxt
        if moved < tol:
            break
    bounds = [(cents[k] + cents[k + 1]) / 2.0 for k in range(levels - 1)]
    return (torch.tensor(cents, dtype=torch.float32),
            torch.tensor(bounds, dtype=torch.float32))


class LloydMaxCodebook:
    """CPU codebook with a process-wide cache (API of lloyd_max.py:107-160)."""

    _cpu_cache: Dict[tuple, "LloydMaxCodebook"] = {}

    def __init__(self, d: int, bits: int, use_exact_pdf: bool = False):
        self.d = d
        self.bits = bits
        self.n_levels = 2 ** bits
        self.centroids, self.boundaries = solve_lloyd_max(d, bits, use_exact_pdf)

    @classmethod
    def get(cls, d: int, bits: int) -> "LloydMaxCodebook":
        key = (d, bits)
        if key not in cls._cpu_cache:
            cls._cpu_cache[key] = cls(d, bits)
        return cls._cpu_cache[key]

    def quantize(self, x: torch.Tensor) -> torch.Tensor:
        """Nearest centroid (argmin), int16 — the legacy slow path."""
        c = self.centroids.to(x.device)
        return (x.unsqueeze(-1) - c).abs().argmin(dim=-1).to(torch.int16)

    def dequantize(self, indices: torch.Tensor) -> torch.Tensor:
        return self.centroids.to(indices.device)[indices.long()]

    def __repr__(self) -> str:
        return f"LloydMaxCodebook(d={self.d}, bits={self.bits}, levels={self.n_levels})"
