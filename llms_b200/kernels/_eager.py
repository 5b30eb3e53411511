"""Small eager helpers used by the drop-in modules around the fused kernels.

The modules keep the engine's behaviour for everything that is not a fused
projection (QK-norm, RoPE, cache writes, SDPA).  These helpers restate the
engine's conventions: RMSNorm computes in fp32, casts back to the input dtype
and then multiplies by the weight (engine/attention.py:20-33); RoPE uses the
"concat" convention with rotate-half (engine/attention.py:36-76).
"""

from __future__ import annotations

import torch
from torch import nn


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return weight * xf.to(x.dtype)


class RMSNorm(nn.Module):
    """Parameter-compatible with the engine's RMSNorm (``weight``, ``eps``;
    engine/attention.py:20-33); forward is :func:`rms_norm`."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: (B, H, T, R); cos/sin: (T, R)."""
    return x * cos[None, None] + rotate_half(x) * sin[None, None]


def norm_module(mod, x: torch.Tensor) -> torch.Tensor:
    """Apply an engine RMSNorm module (anything with ``weight`` and ``eps``)."""
    return rms_norm(x, mod.weight, mod.eps)
