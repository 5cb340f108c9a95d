"""CPU restatement of compress-on-emit (HCA / CSA).  TEST ORACLE ONLY.

Follows aether_2b/serving.py of the reference, in float32 torch:
  * ``emit``  -- _hca_emit :495-505 (softmax over the 128 buffered rows per
                 channel, bias already in z) and the main / index halves of
                 _emit_csa_block :540-575 (rows = [this block's a half ;
                 previous block's b half], a zero / -inf b half for the first
                 block, biases added to z), then
               * RoPE on the last rope_dim channels in interleaved pairs at
                 the given position (modeling.py:122-155: cos / sin of
                 position * inv_freq, repeat-interleaved), main stream only
               * RMSNorm (modeling.py:32-41, F.rms_norm), main stream only
               * PolarQuant encode (``oracle.turboquant.encode``)
Parity with the reference methods themselves is pinned by the ``emit*``
vectors in tests/golden/reference_vectors.npz.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import turboquant as tq


def pool_block(c0: torch.Tensor, z0: torch.Tensor, bias0: Optional[torch.Tensor] = None,
               c1: Optional[torch.Tensor] = None, z1: Optional[torch.Tensor] = None,
               bias1: Optional[torch.Tensor] = None, has1: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gated softmax pooling: c*/z* [B, m, d] -> [B, d] (fp32)."""
    c0, z0 = c0.float(), z0.float()
    if bias0 is not None:
        z0 = z0 + bias0.float()
    if c1 is None:
        c, z = c0, z0
    else:
        c1, z1 = c1.float(), z1.float()
        if bias1 is not None:
            z1 = z1 + bias1.float()
        if has1 is not None:
            keep = has1.view(-1, 1, 1).bool()
            c1 = torch.where(keep, c1, torch.zeros_like(c1))
            z1 = torch.where(keep, z1, torch.full_like(z1, float("-inf")))
        c, z = torch.cat([c0, c1], dim=1), torch.cat([z0, z1], dim=1)
    w = torch.softmax(z, dim=1)
    return (w * c).sum(dim=1)


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate the last 2*len(inv_freq) channels of x [B, d] at positions [B]."""
    r = 2 * inv_freq.numel()
    if r == 0:
        return x
    keep, part = x[..., :-r], x[..., -r:]
    ang = positions.float().unsqueeze(-1) * inv_freq.float()
    cos = torch.repeat_interleave(ang.cos(), 2, dim=-1)
    sin = torch.repeat_interleave(ang.sin(), 2, dim=-1)
    rot = torch.stack((-part[..., 1::2], part[..., 0::2]), dim=-1).flatten(-2)
    return torch.cat([keep, part * cos + rot * sin], dim=-1)


def emit(c0, z0, bias0=None, c1=None, z1=None, bias1=None, has1=None, positions=None, inv_freq=None,
         norm_weight=None, norm_eps: float = 1e-6, bits: Optional[int] = None,
         seed: int = 42) -> Tuple[torch.Tensor, Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Returns (entry fp32 [B, d], codes, scale); codes / scale None without bits.

    One sequence at a time, as the reference emits (torch's CPU reductions
    may round differently for another batch shape)."""
    one = lambda t, b: None if t is None else t[b: b + 1]
    x = torch.cat([pool_block(one(c0, b), one(z0, b), bias0, one(c1, b), one(z1, b), bias1, one(has1, b))
                   for b in range(c0.shape[0])], dim=0)
    if inv_freq is not None:
        x = rope(x, positions, inv_freq)
    if norm_weight is not None:
        x = torch.nn.functional.rms_norm(x, (x.shape[-1],), norm_weight.float(), norm_eps)
    if bits is None:
        return x, None, None
    codes, scale = tq.encode(x, bits, seed)
    return x, codes, scale
