"""Lloyd-Max scalar codebooks for N(0, 1): the alternative TurboQuant level
format (256 levels for 8-bit, 16 for 4-bit).

Lloyd's algorithm (S. P. Lloyd, "Least squares quantization in PCM", 1982;
J. Max, "Quantizing for minimum distortion", 1960): starting from uniform
levels, alternate (a) decision thresholds at the midpoints of adjacent
levels and (b) each level at the conditional mean of N(0, 1) between its
thresholds, E[X | a < X < b] = (phi(a) - phi(b)) / (Phi(b) - Phi(a)), until
the levels stop moving.  The levels are symmetric about 0.

A vector is coded with scale = max|y| / c_max (c_max the largest level), so
y / scale lies in [-c_max, c_max], and each element takes the index of the
nearest level (the lower index on an exact midpoint: the number of
thresholds strictly below the value).  The fp32 threshold table drives both
the kernels and the test oracle, so codes agree bit for bit.
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Tuple

import torch


def _pdf(x: float) -> float:
    return math.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)


def _cdf(x: float) -> float:
    return 0.5 * (1.0 + math.erf(x / math.sqrt(2.0)))


@lru_cache(maxsize=None)
def lloyd_max_levels(levels: int, iters: int = 2000, tol: float = 1e-12) -> Tuple[float, ...]:
    """The `levels` reconstruction levels (ascending, float64) for N(0, 1)."""
    if levels < 2:
        raise ValueError("need at least 2 levels")
    c = [-3.0 + 6.0 * (i + 0.5) / levels for i in range(levels)]
    for _ in range(iters):
        t = [(c[i] + c[i + 1]) / 2.0 for i in range(levels - 1)]
        edges = [-math.inf] + t + [math.inf]
        new = []
        for i in range(levels):
            a, b = edges[i], edges[i + 1]
            pa = 0.0 if a == -math.inf else _pdf(a)
            pb = 0.0 if b == math.inf else _pdf(b)
            mass = (1.0 if b == math.inf else _cdf(b)) - (0.0 if a == -math.inf else _cdf(a))
            new.append((pa - pb) / mass if mass > 0 else c[i])
        # symmetrise (the fixed point is symmetric; this removes drift)
        new = [(new[i] - new[levels - 1 - i]) / 2.0 for i in range(levels)]
        delta = max(abs(x - y) for x, y in zip(new, c))
        c = new
        if delta < tol:
            break
    return tuple(c)


def codebook(bits: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(levels fp32 [2^bits], thresholds fp32 [2^bits - 1]) on the CPU.  The
    thresholds are the fp32 midpoints of adjacent fp32 levels."""
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    lv = torch.tensor(lloyd_max_levels(1 << bits), dtype=torch.float32)
    th = (lv[:-1] + lv[1:]) * 0.5
    return lv, th


_DEV_CACHE = {}


def device_codebook(bits: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    key = (bits, str(device))
    if key not in _DEV_CACHE:
        lv, th = codebook(bits)
        _DEV_CACHE[key] = (lv.to(device), th.to(device))
    return _DEV_CACHE[key]
