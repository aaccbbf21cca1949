"""Lloyd-Max scalar codebook for rotated unit-vector coordinates.

After a random orthogonal rotation, each coordinate of a d-dimensional unit
vector is approximately N(0, 1/d).  The codebook is the Lloyd-Max optimum for
that Gaussian: alternate (1) decision boundaries at midpoints of adjacent
centroids and (2) centroids at the conditional mean of each cell, with the
integrals done by the trapezoid rule on 200 panels over [-10.5 sigma,
10.5 sigma] for the outer cells, starting from uniform centroids on
[-3.5 sigma, 3.5 sigma], stopping after 200 iterations or a 1e-10 change.

This is the procedure of reference/centroids.py:31-86 (same initialisation,
integration rule and stopping rule, so the fp32 centroids agree to the last
bit); it runs once on the host and is cached.
"""

from __future__ import annotations

import math
from functools import lru_cache

import torch


def _gauss(x: float, var: float) -> float:
    # Same float64 operation order as the reference so the fp32 codebook is
    # bit-identical.
    return (1.0 / math.sqrt(2 * math.pi * var)) * math.exp(-x * x / (2 * var))


def _trapezoid(f, a: float, b: float, panels: int = 200) -> float:
    h = (b - a) / panels
    total = 0.5 * (f(a) + f(b))
    for i in range(1, panels):
        total += f(a + i * h)
    return total * h


def solve_lloyd_max(d: int, bits: int, max_iter: int = 200, tol: float = 1e-10):
    """Return ``(centroids, boundaries)`` as fp32 tensors (sorted)."""
    levels = 1 << bits
    var = 1.0 / d
    sigma = math.sqrt(var)
    lo, hi = -3.5 * sigma, 3.5 * sigma
    cents = [lo + (hi - lo) * (i + 0.5) / levels for i in range(levels)]

    def pdf(x):
        return _gauss(x, var)

    def xpdf(x):
        return x * _gauss(x, var)

    for _ in range(max_iter):
        mids = [(cents[i] + cents[i + 1]) / 2.0 for i in range(levels - 1)]
        edges = [3.0 * lo] + mids + [3.0 * hi]
        new = []
        for i in range(levels):
            mass = _trapezoid(pdf, edges[i], edges[i + 1])
            new.append(_trapezoid(xpdf, edges[i], edges[i + 1]) / mass if mass > 1e-15 else cents[i])
        done = max(abs(a - b) for a, b in zip(new, cents)) < tol
        if done:
            break
        cents = new
    mids = [(cents[i] + cents[i + 1]) / 2.0 for i in range(levels - 1)]
    return torch.tensor(cents, dtype=torch.float32), torch.tensor(mids, dtype=torch.float32)


@lru_cache(maxsize=32)
def get_centroids(d: int, bits: int) -> torch.Tensor:
    """fp32 ``[2**bits]`` Lloyd-Max centroids for N(0, 1/d) (cached)."""
    return solve_lloyd_max(d, bits)[0]


def get_midpoints(centroids: torch.Tensor) -> torch.Tensor:
    """Store-side decision boundaries, computed in fp32 from the fp32
    centroids as the reference launchers do
    (reference/turboquant_attn.py:485-486)."""
    c = centroids.float()
    return ((c[:-1] + c[1:]) * 0.5).contiguous()


def build_pair_lut(centroids: torch.Tensor) -> torch.Tensor:
    """``[n*n, 2]`` table with entry ``lo*n + hi = (c[lo], c[hi])``
    (baseline/common.py:232-257).  Accepted by the V2-style launcher for
    interface parity; the sm_100a kernel builds its own table."""
    n = centroids.numel()
    c = centroids.float()
    lut = torch.empty(n, n, 2, dtype=torch.float32, device=centroids.device)
    lut[:, :, 0] = c[:, None]
    lut[:, :, 1] = c[None, :]
    return lut.reshape(n * n, 2).contiguous()
