"""Host-side RoPE / YaRN helpers (the A10 scalars of the decode path).

Restates aether_2b/modeling.py of the reference:
  * ``get_rope_freqs``       :60-99   base 1/theta^(i/half), optional linear or
                                      YaRN blend between base and base/factor
  * ``rope_attention_scale`` :102-109 1 + ln(factor) * yarn_mscale under YaRN
  * ``apply_rope``           :122-155 rotation of the last ``rope_dim`` dims in
                                      interleaved pairs (x[2i], x[2i+1])
The kernels only see the resulting ``softmax_scale``; these helpers build
rotated synthetic inputs and let callers reproduce the model's positions.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class RopeConfig:
    rope_dim: int = 64
    rope_theta: float = 10000.0
    rope_scaling_type: str = "none"
    rope_scaling_factor: float = 1.0
    max_position_embeddings: int = 65536
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    yarn_mscale: float = 0.1

    @classmethod
    def yarn(cls, factor: float, **kw) -> "RopeConfig":
        return cls(rope_scaling_type="yarn", rope_scaling_factor=factor, **kw)


def get_rope_freqs(cfg: RopeConfig, device: Optional[torch.device] = None) -> torch.Tensor:
    rope_dim = cfg.rope_dim - (cfg.rope_dim % 2)
    if rope_dim <= 0:
        return torch.empty(0, device=device, dtype=torch.float32)
    half = rope_dim // 2
    idx = torch.arange(half, device=device, dtype=torch.float32)
    base = 1.0 / (cfg.rope_theta ** (idx / half))
    kind = (cfg.rope_scaling_type or "none").lower()
    factor = max(float(cfg.rope_scaling_factor), 1.0)
    if kind == "linear" and factor > 1.0:
        return base / factor
    if kind != "yarn" or factor <= 1.0:
        return base
    ctx = max(float(cfg.max_position_embeddings), 1.0)
    beta_fast = max(float(cfg.yarn_beta_fast), 1.0)
    beta_slow = max(float(cfg.yarn_beta_slow), 1e-6)
    wavelen = (2.0 * math.pi) / base.clamp_min(1e-12)
    scaled = base / factor
    keep = wavelen <= ctx / beta_fast
    full = wavelen >= ctx / beta_slow
    blend = ~(keep | full)
    if not blend.any():
        return torch.where(keep, base, scaled)
    ramp = ((ctx / wavelen - beta_slow) / max(beta_fast - beta_slow, 1e-6)).clamp(0.0, 1.0)
    mixed = scaled * (1.0 - ramp) + base * ramp
    return torch.where(keep, base, torch.where(full, scaled, mixed))


def rope_attention_scale(cfg: RopeConfig) -> float:
    if (cfg.rope_scaling_type or "none").lower() != "yarn":
        return 1.0
    factor = max(float(cfg.rope_scaling_factor), 1.0)
    if factor <= 1.0:
        return 1.0
    return 1.0 + math.log(factor) * float(cfg.yarn_mscale)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cfg: RopeConfig) -> torch.Tensor:
    """Rotate the last ``rope_dim`` dims of x [..., S, D] (or [..., S, H, D]
    when ``positions`` has one entry per S) at the given positions."""
    rope_dim = min(cfg.rope_dim, x.size(-1))
    rope_dim -= rope_dim % 2
    if rope_dim <= 0:
        return x
    freqs = get_rope_freqs(cfg, device=x.device)[: rope_dim // 2]
    ang = positions.to(x.device).float().unsqueeze(-1) * freqs  # [S, half]
    cos = ang.cos().repeat_interleave(2, dim=-1)
    sin = ang.sin().repeat_interleave(2, dim=-1)
    extra = x.dim() - 1 - positions.dim()  # dims between positions and D (e.g. heads)
    for _ in range(max(extra, 0)):
        cos = cos.unsqueeze(-2)
        sin = sin.unsqueeze(-2)
    xf = x.float()
    keep, rot = xf[..., :-rope_dim], xf[..., -rope_dim:]
    pairs = rot.reshape(*rot.shape[:-1], rope_dim // 2, 2)
    swapped = torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).reshape(rot.shape)
    return torch.cat([keep, rot * cos + swapped * sin], dim=-1).to(x.dtype)
