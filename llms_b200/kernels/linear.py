"""Output (``o``) and down projections on the B200 projection kernels.

The reference engine runs these two bias-free ``nn.Linear`` layers through
cuBLAS: ``self.o(attn)`` (``src/engine/attention.py:163``) and
``self.down(...)`` (``src/engine/model.py:37``).  Here they go through
``b200mm_linear`` / ``b200mm_linear_w8`` in ``libb200mm.so``, which share
the dispatch of the fused QKV projection: the 16-byte-streaming GEMV at
decode batch sizes, the tensor-core GEMVs for small batches and the tcgen05
GEMM for prefill.

:class:`B200Linear` keeps the ``weight`` parameter name of ``nn.Linear`` so
state dicts load unchanged; :class:`Int8Linear` holds per-output-row int8
weights (``qweight``, ``scale``) made by :func:`quantize_per_row`.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _capi
from .quant import quantize_per_row


def _rows(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _check_linear(x: torch.Tensor, W: torch.Tensor) -> None:
    if W.dim() != 2:
        raise ValueError(f"W must be 2D (N, K), got shape {tuple(W.shape)}")
    if x.shape[-1] != W.shape[1]:
        raise ValueError(f"x last dim {x.shape[-1]} != W.shape[1] {W.shape[1]}")
    if x.device != W.device:
        raise ValueError(f"x ({x.device}) and W ({W.device}) must be on the same device")


def b200_linear(x: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """``x @ W.T`` (``F.linear`` without bias) in one sm_100a launch.

    Args:
        x: ``(..., K)``; float32, float16 or bfloat16 on a CUDA device.
        W: ``(N, K)`` in ``nn.Linear.weight`` layout, same dtype and device.

    Returns:
        ``(..., N)`` tensor with ``x``'s dtype and device.
    """
    _check_linear(x, W)
    if x.dtype != W.dtype:
        raise ValueError(f"x ({x.dtype}) and W ({W.dtype}) must share a dtype")
    N, K = W.shape
    lead = x.shape[:-1]
    x2 = _rows(x.reshape(-1, K))
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0 or N == 0:
        return y.reshape(*lead, N)
    if K == 0:
        return y.zero_().reshape(*lead, N)
    _capi.require_cuda(x)
    W2 = _rows(W)
    with _capi.on_device(x):
        st = _capi.lib.b200mm_linear(
            x2.data_ptr(), x2.stride(0), W2.data_ptr(), W2.stride(0), y.data_ptr(), y.stride(0),
            M, N, K, _capi.dtype_code(x.dtype), _capi.stream_of(x),
        )
    _capi.check(st, "b200mm_linear")
    return y.reshape(*lead, N)


def int8_linear(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """``x @ (q * s[:, None]).T`` with int8 ``q`` (N, K) and fp32 ``s`` (N,);
    x is float16 or bfloat16, the output has x's dtype."""
    _check_linear(x, q)
    if q.dtype != torch.int8:
        raise ValueError(f"q must be int8, got {q.dtype}")
    if s.dtype != torch.float32 or s.shape != (q.shape[0],):
        raise ValueError(f"s must be float32 of shape ({q.shape[0]},), got {s.dtype} {tuple(s.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"int8 weights need float16 or bfloat16 activations, got {x.dtype}")
    N, K = q.shape
    lead = x.shape[:-1]
    x2 = _rows(x.reshape(-1, K))
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0 or N == 0:
        return y.reshape(*lead, N)
    if K == 0:
        return y.zero_().reshape(*lead, N)
    _capi.require_cuda(x)
    q2, s2 = _rows(q), s.contiguous()
    with _capi.on_device(x):
        st = _capi.lib.b200mm_linear_w8(
            x2.data_ptr(), x2.stride(0), q2.data_ptr(), s2.data_ptr(), q2.stride(0),
            y.data_ptr(), y.stride(0), M, N, K, _capi.dtype_code(x.dtype), _capi.stream_of(x),
        )
    _capi.check(st, "b200mm_linear_w8")
    return y.reshape(*lead, N)


class B200Linear(nn.Module):
    """Bias-free ``nn.Linear`` whose forward is :func:`b200_linear`."""

    def __init__(self, in_features: int, out_features: int) -> None:
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "B200Linear":
        """Wrap ``lin`` sharing its weight (no copy); ``lin`` must have no bias."""
        if lin.bias is not None:
            raise ValueError("B200Linear serves bias-free projections only")
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        out.in_features, out.out_features = lin.in_features, lin.out_features
        out.weight = lin.weight
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return b200_linear(x, self.weight)


class Int8Linear(nn.Module):
    """Bias-free projection with int8 weight-only storage (buffers
    ``qweight`` [N, K] int8 and ``scale`` [N] fp32)."""

    def __init__(self, in_features: int, out_features: int) -> None:
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("qweight", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(out_features))

    @classmethod
    def from_linear(cls, lin: nn.Module) -> "Int8Linear":
        if getattr(lin, "bias", None) is not None:
            raise ValueError("Int8Linear serves bias-free projections only")
        W = lin.weight
        out = cls(W.shape[1], W.shape[0])
        q, s = quantize_per_row(W)
        out.qweight = q.to(W.device)
        out.scale = s.to(W.device)
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return int8_linear(x, self.qweight, self.scale)
