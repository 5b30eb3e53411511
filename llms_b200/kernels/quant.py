"""Int8 weight-only projections (new in this build; the reference has none).

Weights are stored as int8 ``q`` in [-127, 127] with one fp32 scale per
output row, ``W[n, k] = q[n, k] * s[n]``.  Activations and outputs stay in
the model dtype (bf16/fp16); the kernels dequantise in registers and
accumulate in fp32, so the only difference from the dense path is the weight
rounding done once by :func:`quantize_per_row`.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _capi
from .fused_qkv import TritonAttention


def quantize_per_row(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8: ``s = max|W_row| / 127``,
    ``q = clamp(round(W / s), -127, 127)``.  All-zero rows get ``s = 1``."""
    Wf = W.detach().float()
    amax = Wf.abs().amax(dim=1)
    s = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.clamp(torch.round(Wf / s[:, None]), -127, 127).to(torch.int8)
    return q.contiguous(), s.contiguous()


def dequantize_per_row(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return q.float() * s.float()[:, None]


def _check_w8(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, name: str) -> None:
    if q.dim() != 2 or q.dtype != torch.int8:
        raise ValueError(f"{name} must be a 2D int8 tensor, got {q.dtype} {tuple(q.shape)}")
    if s.dim() != 1 or s.shape[0] != q.shape[0] or s.dtype != torch.float32:
        raise ValueError(f"{name} scales must be float32 of shape ({q.shape[0]},), got {s.dtype} {tuple(s.shape)}")
    if x.shape[-1] != q.shape[1]:
        raise ValueError(f"x last dim {x.shape[-1]} != {name}.shape[1] {q.shape[1]}")
    if x.device != q.device or x.device != s.device:
        raise ValueError(f"x ({x.device}), {name} ({q.device}), scales ({s.device}) must be on the same device")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"int8 weight-only kernels take bfloat16/float16 activations, got {x.dtype}")


def int8_fused_gate_up_silu(x: torch.Tensor, qg: torch.Tensor, sg: torch.Tensor,
                            qu: torch.Tensor, su: torch.Tensor) -> torch.Tensor:
    """``silu((x qg^T) sg) * ((x qu^T) su)``; shapes as ``triton_fused_gate_up_silu``."""
    if qg.shape != qu.shape:
        raise ValueError(f"Wg shape {tuple(qg.shape)} != Wu shape {tuple(qu.shape)}")
    _check_w8(x, qg, sg, "Wg")
    _check_w8(x, qu, su, "Wu")
    N, K = qg.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M and N:
        _capi.require_cuda(x)
        qg2, qu2 = qg.contiguous(), qu.contiguous()
        with _capi.on_device(x):
            st = _capi.lib.b200mm_gate_up_silu_w8(
                x2.data_ptr(), x2.stride(0), qg2.data_ptr(), sg.data_ptr(), qu2.data_ptr(),
                su.data_ptr(), qg2.stride(0), y.data_ptr(), y.stride(0), M, N, K,
                _capi.dtype_code(x.dtype), _capi.stream_of(x),
            )
        _capi.check(st, "b200mm_gate_up_silu_w8")
    return y.reshape(*lead, N)


def int8_fused_qkv(x: torch.Tensor, q_qkv: torch.Tensor, s_qkv: torch.Tensor, *, n_q: int, n_k: int):
    """``split((x q_qkv^T) * s_qkv)`` into q/k/v views; shapes as ``triton_fused_qkv``."""
    _check_w8(x, q_qkv, s_qkv, "W_qkv")
    n_total, K = q_qkv.shape
    if n_q + 2 * n_k != n_total:
        raise ValueError(f"n_q + 2*n_k ({n_q} + 2*{n_k} = {n_q + 2 * n_k}) != W_qkv.shape[0] ({n_total})")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty((M, n_total), dtype=x.dtype, device=x.device)
    if M and n_total:
        _capi.require_cuda(x)
        W = q_qkv if q_qkv.stride(-1) == 1 else q_qkv.contiguous()
        with _capi.on_device(x):
            st = _capi.lib.b200mm_qkv_w8(
                x2.data_ptr(), x2.stride(0), W.data_ptr(), s_qkv.data_ptr(), W.stride(0),
                y.data_ptr(), y.stride(0), M, n_total, K,
                _capi.dtype_code(x.dtype), _capi.stream_of(x),
            )
        _capi.check(st, "b200mm_qkv_w8")
    y = y.reshape(*lead, n_total)
    return y.split([n_q, n_k, n_k], dim=-1)


class Int8FFN(nn.Module):
    """SwiGLU FFN with int8 weight-only gate/up (buffers ``qg, sg, qu, su``);
    ``down`` stays a dense ``nn.Linear``."""

    def __init__(self, hidden_size: int, intermediate_size: int) -> None:
        super().__init__()
        self.register_buffer("qg", torch.zeros(intermediate_size, hidden_size, dtype=torch.int8))
        self.register_buffer("sg", torch.ones(intermediate_size))
        self.register_buffer("qu", torch.zeros(intermediate_size, hidden_size, dtype=torch.int8))
        self.register_buffer("su", torch.ones(intermediate_size))
        self.down = nn.Linear(intermediate_size, hidden_size, bias=False)

    @classmethod
    def from_eager(cls, eager: nn.Module) -> "Int8FFN":
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        qg, sg = quantize_per_row(eager.gate.weight)
        qu, su = quantize_per_row(eager.up.weight)
        for name, t in (("qg", qg), ("sg", sg), ("qu", qu), ("su", su)):
            out.register_buffer(name, t.to(eager.gate.weight.device))
        out.down = eager.down
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(int8_fused_gate_up_silu(x, self.qg, self.sg, self.qu, self.su))


class Int8Attention(TritonAttention):
    """``TritonAttention`` whose fused QKV projection reads int8 weights
    (buffers ``q_qkv``, ``s_qkv``) instead of a dense ``W_qkv``."""

    def __init__(self, *, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 rms_eps: float) -> None:
        super().__init__(hidden_size=hidden_size, num_heads=num_heads, num_kv_heads=num_kv_heads,
                         head_dim=head_dim, rms_eps=rms_eps)
        del self.W_qkv
        n_total = self.n_q + 2 * self.n_k
        self.register_buffer("q_qkv", torch.zeros(n_total, hidden_size, dtype=torch.int8))
        self.register_buffer("s_qkv", torch.ones(n_total))

    @classmethod
    def from_eager(cls, eager: nn.Module) -> "Int8Attention":
        """From an engine ``Attention`` (q/k/v Linears) or a ``TritonAttention``."""
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        if hasattr(eager, "W_qkv"):
            W = eager.W_qkv
            out.hidden_size = W.shape[1]
        else:
            W = torch.cat([eager.q.weight, eager.k.weight, eager.v.weight], dim=0)
            out.hidden_size = eager.q.in_features
        out.num_heads = eager.num_heads
        out.num_kv_heads = eager.num_kv_heads
        out.head_dim = eager.head_dim
        out.n_q = eager.num_heads * eager.head_dim
        out.n_k = eager.num_kv_heads * eager.head_dim
        q, s = quantize_per_row(W)
        out.register_buffer("q_qkv", q.to(W.device))
        out.register_buffer("s_qkv", s.to(W.device))
        out.o = eager.o
        out.q_norm = eager.q_norm
        out.k_norm = eager.k_norm
        out.decode_attn_op = getattr(eager, "decode_attn_op", None)
        return out

    def project_qkv(self, x: torch.Tensor):
        return int8_fused_qkv(x, self.q_qkv, self.s_qkv, n_q=self.n_q, n_k=self.n_k)
