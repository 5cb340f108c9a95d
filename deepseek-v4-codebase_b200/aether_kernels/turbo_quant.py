"""PolarQuant API of the reference (aether_2b/turbo_quant.py:79-211) backed by
the sm_100a kernels.  Encode is bit-identical to the reference's fp32 torch
path; decode matches it to fp32 rounding of the final cast.

Tensors must live on a CUDA device: there is no CPU implementation here.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import ops


def _wht(x: torch.Tensor) -> torch.Tensor:
    """Normalised Walsh-Hadamard transform on the last dim (fp32 result)."""
    d = x.shape[-1]
    if d == 0 or (d & (d - 1)) != 0:
        raise ValueError(f"WHT requires last dim to be a power of 2, got {d}")
    if not x.is_cuda:
        raise RuntimeError("aether_kernels.turbo_quant._wht requires a CUDA tensor")
    return ops.wht(x)


class PolarQuant:
    """Randomised Hadamard rotation + symmetric per-vector scalar quantization.

    bits=8 -> int8 codes [..., D]; bits=4 -> uint8 [..., D/2] with two signed
    4-bit codes per byte (even index in the low nibble).  Scale fp32 [..., 1].

    ``codebook="lloyd-max"`` (not in the reference) selects the Lloyd-Max
    level format for N(0, 1) instead of the uniform levels: codes are level
    indices (uint8 [..., D], or index nibbles [..., D/2]).  A
    ``TurboQuantPagedCache(..., codebook="lloyd-max")`` holds pages in this
    format and the fused paged decode kernels apply the level table
    themselves (the prefill indexer and compress-on-emit write / read the
    uniform format only).
    """

    def __init__(self, bits: int, seed: int = 42, codebook: str = "uniform") -> None:
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        if codebook not in ("uniform", "lloyd-max"):
            raise ValueError(f"codebook must be 'uniform' or 'lloyd-max', got {codebook!r}")
        self.codebook = codebook
        self.bits = bits
        self._seed = seed
        self._diag_cache: Dict[Tuple[int, str], torch.Tensor] = {}

    def _diag(self, d: int, device: torch.device) -> torch.Tensor:
        key = (d, str(device))
        if key not in self._diag_cache:
            self._diag_cache[key] = ops.rademacher_diag(d, self._seed, torch.device(device))
        return self._diag_cache[key]

    def encode(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        if not x.is_cuda:
            raise RuntimeError("aether_kernels PolarQuant.encode requires a CUDA tensor")
        if self.codebook == "lloyd-max":
            return ops.tq_encode_lut(x.contiguous(), self.bits, self._seed)
        return ops.tq_encode(x.contiguous(), self.bits, self._seed)

    def decode(self, data: torch.Tensor, scale: torch.Tensor,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        if not data.is_cuda:
            raise RuntimeError("aether_kernels PolarQuant.decode requires a CUDA tensor")
        if self.codebook == "lloyd-max":
            return ops.tq_decode_lut(data.contiguous(), scale, self.bits, self._seed, out_dtype)
        return ops.tq_decode(data.contiguous(), scale, self.bits, self._seed, out_dtype)
