"""CPU restatement of TurboQuant (PolarQuant) encode / decode.  TEST ORACLE ONLY.

Follows aether_2b/turbo_quant.py of the reference:
  * ``wht``          -- :49-76   fp32 radix-2 butterfly, stages h = 1, 2, 4, ...
                                 each stage maps a block [a | b] of width 2h to
                                 [a + b | a - b]; the result is scaled by d**-0.5
  * ``rademacher``   -- :111-121 CPU torch.Generator seeded seed*10007 + d,
                                 sign = +1 where torch.rand(d) > 0.5
  * ``encode``       -- :127-166 y = WHT(diag * x); per-vector absmax m
                                 (clamped to 1e-8); code = clamp(round(y / m * L))
                                 with L = 127 (int8) or 7 (packed signed nibbles,
                                 even index in the low nibble); scale = m / L
  * ``decode``       -- :168-211 x = WHT(code * scale) * diag

The arithmetic is float32 torch on the CPU in the same op order, so the codes
match the reference bit for bit (checked against golden vectors).
"""
from __future__ import annotations

from typing import Tuple

import torch

LEVELS = {8: 127, 4: 7}


def wht(x: torch.Tensor) -> torch.Tensor:
    """Normalised Walsh-Hadamard transform over the last dim (fp32)."""
    d = x.shape[-1]
    if d == 0 or (d & (d - 1)) != 0:
        raise ValueError(f"WHT requires last dim to be a power of 2, got {d}")
    lead = x.shape[:-1]
    y = x.to(torch.float32).clone()
    h = 1
    while h < d:
        blk = y.reshape(*lead, d // (2 * h), 2, h)
        lo = blk[..., 0, :]
        hi = blk[..., 1, :]
        y = torch.stack([lo + hi, lo - hi], dim=-2).reshape(*lead, d)
        h *= 2
    return y * (d ** -0.5)


def rademacher(d: int, seed: int = 42) -> torch.Tensor:
    """Fixed +-1 diagonal for dimension ``d`` (fp32, CPU)."""
    g = torch.Generator()
    g.manual_seed(seed * 10007 + d)
    r = torch.rand(d, generator=g)
    return torch.where(r > 0.5, torch.ones(d), -torch.ones(d))


def encode(x: torch.Tensor, bits: int, seed: int = 42) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (codes, scale): int8 [...,D] or packed uint8 [...,D/2]; fp32 [...,1]."""
    if bits not in LEVELS:
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    lv = float(LEVELS[bits])
    d = x.shape[-1]
    y = wht(x.float() * rademacher(d, seed))
    m = y.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    scale = m / lv
    q = (y / m * lv).round().clamp(-lv, lv)
    if bits == 8:
        return q.to(torch.int8), scale
    qi = q.to(torch.int32)
    packed = (qi[..., 0::2] & 0xF) | ((qi[..., 1::2] & 0xF) << 4)
    return packed.to(torch.uint8), scale


def unpack_codes(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Signed integer codes [..., D] as fp32 (nibbles sign-extended for 4-bit)."""
    if bits == 8:
        # pools store 8-bit codes as raw bytes; reinterpret as two's complement
        if codes.dtype == torch.uint8:
            codes = codes.view(torch.int8)
        return codes.to(torch.float32)
    c = codes.to(torch.int32)
    lo = c & 0xF
    hi = (c >> 4) & 0xF
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2).to(torch.float32)


def decode(codes: torch.Tensor, scale: torch.Tensor, bits: int, seed: int = 42,
           out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    rot = unpack_codes(codes, bits) * scale.to(torch.float32)
    d = rot.shape[-1]
    return (wht(rot) * rademacher(d, seed)).to(out_dtype)


# ----------------------------------------------------------------------
# Lloyd-Max level format (the alternative to the uniform levels; the
# reference has no such path, so this restates the published algorithm).


def lloyd_max_levels(levels: int, iters: int = 2000) -> torch.Tensor:
    """Lloyd's algorithm for N(0, 1) (Lloyd 1982, Max 1960) in float64:
    thresholds at midpoints, levels at the conditional means
    (phi(a) - phi(b)) / (Phi(b) - Phi(a)); symmetric."""
    import math

    c = torch.tensor([-3.0 + 6.0 * (i + 0.5) / levels for i in range(levels)], dtype=torch.float64)
    n = torch.distributions.Normal(torch.tensor(0.0, dtype=torch.float64), torch.tensor(1.0, dtype=torch.float64))
    for _ in range(iters):
        t = (c[:-1] + c[1:]) / 2
        a = torch.cat([torch.tensor([-math.inf], dtype=torch.float64), t])
        b = torch.cat([t, torch.tensor([math.inf], dtype=torch.float64)])
        pdf = lambda x: torch.where(torch.isinf(x), torch.zeros_like(x), torch.exp(-0.5 * x * x) / math.sqrt(2 * math.pi))
        new = (pdf(a) - pdf(b)) / (n.cdf(b) - n.cdf(a))
        new = (new - new.flip(0)) / 2
        if float((new - c).abs().max()) < 1e-12:
            c = new
            break
        c = new
    return c


def encode_lut(x: torch.Tensor, bits: int, levels: torch.Tensor, seed: int = 42):
    """Codes are the index of the nearest of the fp32 levels (lower index on a
    midpoint) of y / scale, scale = max|y| / max(level), y = WHT(diag * x)."""
    lv = levels.to(torch.float32)
    thr = (lv[:-1] + lv[1:]) * 0.5
    d = x.shape[-1]
    y = wht(x.float() * rademacher(d, seed))
    m = y.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    scale = m / lv[-1]
    u = y / scale
    idx = torch.searchsorted(thr, u.contiguous(), right=False)  # thresholds strictly below u
    if bits == 8:
        return idx.to(torch.uint8), scale
    q = idx.to(torch.int32)
    return ((q[..., 0::2] & 0xF) | ((q[..., 1::2] & 0xF) << 4)).to(torch.uint8), scale


def decode_lut(codes: torch.Tensor, scale: torch.Tensor, bits: int, levels: torch.Tensor, seed: int = 42):
    lv = levels.to(torch.float32)
    if bits == 8:
        idx = codes.to(torch.long)
    else:
        c = codes.to(torch.int32)
        idx = torch.stack([c & 0xF, (c >> 4) & 0xF], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2).long()
    rot = lv[idx] * scale.to(torch.float32)
    return wht(rot) * rademacher(rot.shape[-1], seed)
