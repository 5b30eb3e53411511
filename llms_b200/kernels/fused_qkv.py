"""Fused QKV projection on B200, behind the reference's entry points.

Drop-in for ``kernels/fused_qkv.py`` of the reference engine:
``triton_fused_qkv(x, W_qkv, *, n_q, n_k)`` (reference lines 88-149) and
``TritonAttention`` (reference lines 152-282).  One ``b200mm_qkv`` launch
computes ``x @ W_qkv.T`` into a single ``[M, n_q + 2 n_k]`` buffer; q, k, v
are zero-copy column views of it, as in the reference.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import _capi
from ._eager import RMSNorm, rope
from .glue import fits_qk_norm_rope, qk_norm_rope_cache


def _check_qkv_args(x: torch.Tensor, W_qkv: torch.Tensor, n_q: int, n_k: int) -> None:
    # Same checks, order and messages as reference fused_qkv.py:107-125.
    if W_qkv.dim() != 2:
        raise ValueError(f"W_qkv must be 2D (n_q+2*n_k, K), got shape {tuple(W_qkv.shape)}")
    n_total, K = W_qkv.shape
    if n_q + 2 * n_k != n_total:
        raise ValueError(
            f"n_q + 2*n_k ({n_q} + 2*{n_k} = {n_q + 2 * n_k}) != W_qkv.shape[0] ({n_total})"
        )
    if x.shape[-1] != K:
        raise ValueError(f"x last dim {x.shape[-1]} != W_qkv.shape[1] {K}")
    if x.device != W_qkv.device:
        raise ValueError(f"x ({x.device}) and W_qkv ({W_qkv.device}) must be on the same device")
    if x.dtype != W_qkv.dtype:
        raise ValueError(f"x ({x.dtype}) and W_qkv ({W_qkv.dtype}) must share a dtype")


def triton_fused_qkv(
    x: torch.Tensor, W_qkv: torch.Tensor, *, n_q: int, n_k: int
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(q, k, v) = split(x @ W_qkv.T)`` in one sm_100a kernel launch.

    Args:
        x: ``(..., K)`` on a CUDA device.
        W_qkv: ``(n_q + 2*n_k, K)``, row-stacked ``[Wq; Wk; Wv]``.
        n_q, n_k: rows of the Q block and of each of the K and V blocks.

    Returns:
        ``(q, k, v)`` views of one output buffer, shapes ``(..., n_q)``,
        ``(..., n_k)``, ``(..., n_k)``; dtype and device of ``x``.
    """
    _check_qkv_args(x, W_qkv, n_q, n_k)
    n_total, K = W_qkv.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty((M, n_total), dtype=x.dtype, device=x.device)
    if M > 0 and n_total > 0:
        if K == 0:
            y.zero_()
        else:
            _capi.require_cuda(x)
            W = W_qkv if W_qkv.stride(-1) == 1 else W_qkv.contiguous()
            with _capi.on_device(x):
                st = _capi.lib.b200mm_qkv(
                    x2.data_ptr(), x2.stride(0), W.data_ptr(), W.stride(0),
                    y.data_ptr(), y.stride(0), M, n_total, K,
                    _capi.dtype_code(x.dtype), _capi.stream_of(x),
                )
            _capi.check(st, "b200mm_qkv")
    y = y.reshape(*lead, n_total)
    q, k, v = y.split([n_q, n_k, n_k], dim=-1)
    return q, k, v


def _one_buffer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor | None:
    """The [*, n_q + 2 n_k] buffer q / k / v are split views of (the fused
    projections return such views), or None if they are not adjacent."""
    n_q, n_k = q.shape[-1], k.shape[-1]
    e = q.element_size()
    if (q.stride(-1) != 1 or k.stride() != q.stride() or v.stride() != q.stride()
            or k.data_ptr() != q.data_ptr() + n_q * e or v.data_ptr() != k.data_ptr() + n_k * e):
        return None
    return q.as_strided(q.shape[:-1] + (n_q + 2 * n_k,), q.stride())


class TritonAttention(nn.Module):
    """Drop-in for the engine's GQA ``Attention`` whose q/k/v projections run
    as one fused B200 launch against a pre-concatenated ``W_qkv``.

    QK-norm, RoPE, the KV-cache write and SDPA stay on the engine's eager
    path, exactly as in the reference module (reference fused_qkv.py:228-282).
    """

    def __init__(self, *, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 rms_eps: float) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.n_q = num_heads * head_dim
        self.n_k = num_kv_heads * head_dim
        self.W_qkv = nn.Parameter(torch.empty(self.n_q + 2 * self.n_k, hidden_size), requires_grad=False)
        self.o = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        self.q_norm = RMSNorm(head_dim, eps=rms_eps)
        self.k_norm = RMSNorm(head_dim, eps=rms_eps)
        # the engine Attention's swappable single-query op (engine/attention.py:101-105)
        self.decode_attn_op = None

    @classmethod
    def from_eager(cls, eager: nn.Module) -> "TritonAttention":
        """Build from a loaded engine ``Attention``: concatenates
        ``[Wq; Wk; Wv]`` once and reuses ``o``, ``q_norm``, ``k_norm``."""
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        out.hidden_size = eager.q.in_features
        out.num_heads = eager.num_heads
        out.num_kv_heads = eager.num_kv_heads
        out.head_dim = eager.head_dim
        out.n_q = eager.num_heads * eager.head_dim
        out.n_k = eager.num_kv_heads * eager.head_dim
        W_qkv = torch.cat([eager.q.weight, eager.k.weight, eager.v.weight], dim=0)
        out.W_qkv = nn.Parameter(W_qkv, requires_grad=False)
        out.o = eager.o
        out.q_norm = eager.q_norm
        out.k_norm = eager.k_norm
        out.decode_attn_op = getattr(eager, "decode_attn_op", None)
        return out

    def project_qkv(self, x: torch.Tensor):
        return triton_fused_qkv(x, self.W_qkv, n_q=self.n_q, n_k=self.n_k)

    def forward(self, x: torch.Tensor, *, kv_cache, layer_idx: int, cos: torch.Tensor,
                sin: torch.Tensor, start_pos: int) -> torch.Tensor:
        B, T, _ = x.shape
        qf, kf, vf = self.project_qkv(x)
        end = start_pos + T
        flat = _one_buffer(qf, kf, vf)
        if T == 1 and flat is not None and fits_qk_norm_rope(flat, self.q_norm, self.k_norm, cos, self.head_dim):
            # one launch for q_norm, k_norm, RoPE and the cache write of the
            # decode token (the same rounding as the eager lines below)
            q = qk_norm_rope_cache(flat, self.q_norm, self.k_norm, cos, sin, num_heads=self.num_heads,
                                   num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                                   k_cache=kv_cache.k[layer_idx][:, :, start_pos:],
                                   v_cache=kv_cache.v[layer_idx][:, :, start_pos:], pos=0)
        else:
            q = self.q_norm(qf.view(B, T, self.num_heads, self.head_dim)).transpose(1, 2)
            k = self.k_norm(kf.view(B, T, self.num_kv_heads, self.head_dim)).transpose(1, 2)
            v = vf.view(B, T, self.num_kv_heads, self.head_dim).transpose(1, 2)
            q, k = rope(q, cos, sin), rope(k, cos, sin)
            kv_cache.k[layer_idx][:B, :, start_pos:end, :] = k
            kv_cache.v[layer_idx][:B, :, start_pos:end, :] = v
        full_k = kv_cache.k[layer_idx][:B, :, :end, :]
        full_v = kv_cache.v[layer_idx][:B, :, :end, :]
        op = getattr(self, "decode_attn_op", None)
        if T == 1 and op is not None:  # the engine's decode seam (engine/attention.py:138-145)
            attn = op(q, full_k, full_v, scale=self.head_dim ** -0.5, layer_idx=layer_idx)
            return self.o(attn.transpose(1, 2).reshape(B, T, self.num_heads * self.head_dim))
        rep = self.num_heads // self.num_kv_heads
        if rep > 1:
            full_k = full_k.repeat_interleave(rep, dim=1)
            full_v = full_v.repeat_interleave(rep, dim=1)
        if T == 1:
            attn = F.scaled_dot_product_attention(q, full_k, full_v, is_causal=False)
        elif start_pos == 0:
            attn = F.scaled_dot_product_attention(q, full_k, full_v, is_causal=True)
        else:
            qp = torch.arange(start_pos, end, device=q.device).unsqueeze(1)
            kp = torch.arange(0, end, device=q.device).unsqueeze(0)
            attn = F.scaled_dot_product_attention(q, full_k, full_v, attn_mask=qp >= kp)
        attn = attn.transpose(1, 2).reshape(B, T, self.num_heads * self.head_dim)
        return self.o(attn)
