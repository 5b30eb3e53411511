"""Fused gate-up-SiLU projection on B200, behind the reference's entry points.

Drop-in for ``kernels/fused_ffn.py`` of the reference engine:
``triton_fused_gate_up_silu(x, Wg, Wu)`` (reference lines 98-152) and the
``TritonFFN`` module (reference lines 155-185) keep their names, argument
meaning, output dtype/shape and ``ValueError`` messages.  The work is done by
``b200mm_gate_up_silu`` in ``libb200mm.so``: one launch computes
``silu(x Wg^T) * (x Wu^T)`` with fp32 accumulation, and the [M, 2N]
gate/up intermediate never reaches HBM.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _capi


def _check_gate_up_args(x: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor) -> None:
    # Same checks, order and messages as reference fused_ffn.py:110-124.
    if Wg.shape != Wu.shape:
        raise ValueError(f"Wg shape {tuple(Wg.shape)} != Wu shape {tuple(Wu.shape)}")
    if Wg.dim() != 2:
        raise ValueError(f"Wg must be 2D (N, K), got shape {tuple(Wg.shape)}")
    if x.shape[-1] != Wg.shape[1]:
        raise ValueError(f"x last dim {x.shape[-1]} != Wg.shape[1] {Wg.shape[1]}")
    if x.device != Wg.device or x.device != Wu.device:
        raise ValueError(
            f"x ({x.device}), Wg ({Wg.device}), Wu ({Wu.device}) must be on the same device"
        )
    if not (x.dtype == Wg.dtype == Wu.dtype):
        raise ValueError(f"x ({x.dtype}), Wg ({Wg.dtype}), Wu ({Wu.dtype}) must share a dtype")


def _rows(t: torch.Tensor) -> torch.Tensor:
    """2-D view with unit inner stride (copies only if the last dim is strided)."""
    return t if t.stride(-1) == 1 else t.contiguous()


def triton_fused_gate_up_silu(x: torch.Tensor, Wg: torch.Tensor, Wu: torch.Tensor) -> torch.Tensor:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` in one sm_100a kernel launch.

    Args:
        x: ``(..., K)``; float32, float16 or bfloat16 on a CUDA device.
        Wg, Wu: ``(N, K)`` in ``nn.Linear.weight`` layout, same dtype/device.

    Returns:
        ``(..., N)`` tensor with ``x``'s dtype and device.
    """
    _check_gate_up_args(x, Wg, Wu)
    N, K = Wg.shape
    lead = x.shape[:-1]
    x2 = _rows(x.reshape(-1, K))
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0 or N == 0:
        return y.reshape(*lead, N)
    if K == 0:
        return y.zero_().reshape(*lead, N)
    _capi.require_cuda(x)
    Wg2, Wu2 = _rows(Wg), _rows(Wu)
    with _capi.on_device(x):
        st = _capi.lib.b200mm_gate_up_silu(
            x2.data_ptr(), x2.stride(0),
            Wg2.data_ptr(), Wg2.stride(0),
            Wu2.data_ptr(), Wu2.stride(0),
            y.data_ptr(), y.stride(0),
            M, N, K, _capi.dtype_code(x.dtype), _capi.stream_of(x),
        )
    _capi.check(st, "b200mm_gate_up_silu")
    return y.reshape(*lead, N)


class TritonFFN(nn.Module):
    """Drop-in for the engine's SwiGLU ``FFN`` whose gate/up stage runs the
    fused B200 kernel; ``down`` stays an ``nn.Linear``.

    Parameter names (``gate.weight``, ``up.weight``, ``down.weight``) match
    the engine's ``FFN`` so state dicts load unchanged.
    """

    def __init__(self, hidden_size: int, intermediate_size: int) -> None:
        super().__init__()
        self.gate = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(triton_fused_gate_up_silu(x, self.gate.weight, self.up.weight))

    @classmethod
    def from_eager(cls, eager: nn.Module) -> "TritonFFN":
        """Wrap a module with ``gate``/``up``/``down`` Linears, sharing their
        parameters (no copy)."""
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        out.gate = eager.gate
        out.up = eager.up
        out.down = eager.down
        return out
