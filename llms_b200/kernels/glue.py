"""The decode step's small ops around the projections, each one launch of
this library instead of the engine's chains of elementwise torch kernels.

* :func:`rms_norm` -- the engine's RMSNorm (engine/attention.py:20-33), with
  the residual add before it folded in when ``residual`` is given
  (engine/model.py:54-63), same rounding points (``b200mm_rmsnorm``);
* :func:`qk_norm_rope_cache` -- q_norm, k_norm, RoPE and the KV-cache write
  of one decode token per row, straight from the fused QKV output
  (engine/attention.py:119-131, ``b200mm_qk_norm_rope``).

Both run on CUDA tensors only (no CPU path).  :func:`fits_rms_norm` /
:func:`fits_qk_norm_rope` tell a caller whether a call qualifies, so a
module can keep the engine's own torch ops for what does not (other dtypes
mixed in one call, unaligned rows).
"""

from __future__ import annotations

import torch

from .. import _capi


def _al16(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0 and (t.dim() < 2 or (t.stride(-2) * t.element_size()) % 16 == 0)


def fits_rms_norm(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype in _capi.DTYPE_CODES and weight.dtype == x.dtype and weight.is_contiguous()
            and x.shape[-1] == weight.shape[0] and x.shape[-1] * x.element_size() % 16 == 0
            and x.shape[-1] <= 16384)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """``weight * cast(float(h) * rsqrt(mean(float(h)^2) + eps))`` over the last
    dim, with ``h = x`` or ``h = x + residual`` (rounded to x.dtype).  Returns
    ``y``, or ``(h, y)`` when ``residual`` is given."""
    _capi.require_cuda(x, weight)
    N = x.shape[-1]
    x2 = x.reshape(-1, N)
    if x2.stride(-1) != 1 or not _al16(x2):
        x2 = x2.contiguous()
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, N)
        if r2.stride(-1) != 1 or not _al16(r2):
            r2 = r2.contiguous()
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    h = torch.empty((M, N), dtype=x.dtype, device=x.device) if residual is not None else None
    with _capi.on_device(x):
        st = _capi.lib.b200mm_rmsnorm(
            x2.data_ptr(), x2.stride(0), None if r2 is None else r2.data_ptr(), 0 if r2 is None else r2.stride(0),
            None if h is None else h.data_ptr(), 0 if h is None else h.stride(0), weight.data_ptr(),
            y.data_ptr(), y.stride(0), M, N, float(eps), _capi.dtype_code(x.dtype), _capi.stream_of(x))
    _capi.check(st, "b200mm_rmsnorm")
    y = y.reshape(x.shape)
    return y if h is None else (h.reshape(x.shape), y)


def fits_qk_norm_rope(qkv: torch.Tensor, q_norm, k_norm, cos: torch.Tensor, head_dim: int) -> bool:
    return (qkv.is_cuda and qkv.dtype in _capi.DTYPE_CODES and head_dim in (64, 128, 256)
            and q_norm.weight.dtype == qkv.dtype and k_norm.weight.dtype == qkv.dtype
            and cos.dtype == qkv.dtype and cos.is_contiguous() and q_norm.eps == k_norm.eps)


def qk_norm_rope_cache(qkv: torch.Tensor, q_norm, k_norm, cos_table: torch.Tensor, sin_table: torch.Tensor, *,
                       num_heads: int, num_kv_heads: int, head_dim: int, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, pos: int | torch.Tensor) -> torch.Tensor:
    """One decode token per row: ``qkv`` (B, 1, (H + 2 KV) D) from the fused
    projection; writes rope(k_norm(k)) and v into ``k_cache`` / ``v_cache``
    (B_max, KV, S, D) at ``pos`` and returns rope(q_norm(q)) as (B, H, 1, D).
    ``cos_table`` / ``sin_table`` are the model's whole (max_pos, D) tables in
    the activation dtype; ``pos`` is an int, or a device int64 tensor of one
    element (kept inside the table by the caller)."""
    _capi.require_cuda(qkv, k_cache, v_cache, cos_table)
    B = qkv.shape[0]
    H, KV, D = num_heads, num_kv_heads, head_dim
    q2 = qkv.reshape(B, -1)
    if q2.stride(-1) != 1:
        q2 = q2.contiguous()
    q_out = torch.empty((B, H, 1, D), dtype=qkv.dtype, device=qkv.device)
    dev_pos = isinstance(pos, torch.Tensor)
    for c in (k_cache, v_cache):
        if c.stride(-1) != 1:
            raise ValueError("the KV cache must be contiguous in its last dim")
    with _capi.on_device(qkv):
        st = _capi.lib.b200mm_qk_norm_rope(
            q2.data_ptr(), q2.stride(0), B, H, KV, D, q_norm.weight.data_ptr(), k_norm.weight.data_ptr(),
            cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], 0 if dev_pos else int(pos),
            pos.data_ptr() if dev_pos else None, q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
            k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
            float(q_norm.eps), _capi.dtype_code(qkv.dtype), _capi.stream_of(qkv))
    _capi.check(st, "b200mm_qk_norm_rope")
    return q_out
