"""GQA decode attention on B200, behind the engine's swappable decode op.

The engine's ``Attention`` exposes ``decode_attn_op`` (reference
``src/engine/attention.py:101-105``): when set, the single-query (T == 1)
step calls ``op(q, full_k, full_v, scale=..., layer_idx=...)`` with ``q`` of
shape (B, H, 1, D) and the cache views ``full_k``/``full_v`` of shape
(B, KV, L, D) *before* the GQA expansion (``:138-145``), and expects
(B, H, 1, D) back.  :func:`b200_decode_attn` is such an op: one split-context
kernel streams each (row, KV head) block of the cache once for all g = H / KV
query heads, and a merge kernel combines the partial softmaxes (``b200mm_gqa_decode``).
:func:`apply_decode_attn` installs it on every layer.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _capi

_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """One growing workspace per (device, stream): calls on one stream are
    ordered, so they may share it.  Zero-filled once; each call leaves its
    flag words zeroed for the next."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def b200_decode_attn(q: torch.Tensor, full_k: torch.Tensor, full_v: torch.Tensor, *, scale: float,
                     layer_idx: int | None = None) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` for one query token per row, with K/V shared
    by groups of H / KV query heads.

    Args:
        q: (B, H, 1, D) query (after QK-norm and RoPE).
        full_k, full_v: (B, KV, L, D) cache views; the last dim must be
            contiguous (any other strides are taken as they are).
        scale: softmax scale (the engine passes ``head_dim ** -0.5``).
        layer_idx: accepted for the hook's signature; unused.

    Returns:
        (B, H, 1, D) in ``q``'s dtype.
    """
    del layer_idx
    if q.dim() != 4 or q.shape[2] != 1:
        raise ValueError(f"q must be (B, H, 1, D), got {tuple(q.shape)}")
    if full_k.dim() != 4 or full_k.shape != full_v.shape:
        raise ValueError(f"full_k {tuple(full_k.shape)} and full_v {tuple(full_v.shape)} must be the same (B, KV, L, D)")
    B, H, _, D = q.shape
    Bk, KV, L, Dk = full_k.shape
    if Bk != B or Dk != D or KV < 1 or H % KV:
        raise ValueError(f"q {tuple(q.shape)} does not match the cache views {tuple(full_k.shape)}")
    if not (q.dtype == full_k.dtype == full_v.dtype):
        raise ValueError(f"q ({q.dtype}), full_k ({full_k.dtype}), full_v ({full_v.dtype}) must share a dtype")
    _capi.require_cuda(q, full_k, full_v)
    out = torch.empty((B, H, 1, D), dtype=q.dtype, device=q.device)
    if B == 0:
        return out
    if L == 0:
        raise ValueError("the cache views hold no tokens")
    qq = q if q.stride(-1) == 1 else q.contiguous()
    k = full_k if full_k.stride(-1) == 1 else full_k.contiguous()
    v = full_v if full_v.stride(-1) == 1 else full_v.contiguous()
    with _capi.on_device(q):
        stream = _capi.stream_of(q)
        need = _capi.lib.b200mm_gqa_decode_workspace_size(B, H, KV, D, L)
        if need == 0:
            raise ValueError(f"unsupported GQA decode shape B={B} H={H} KV={KV} D={D} L={L}")
        ws = _workspace(q.device, stream, need)
        st = _capi.lib.b200mm_gqa_decode(
            qq.data_ptr(), qq.stride(0), qq.stride(1),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
            out.data_ptr(), out.stride(0), out.stride(1),
            B, H, KV, D, L, float(scale), _capi.dtype_code(q.dtype),
            ws.data_ptr(), ws.numel(), stream,
        )
    _capi.check(st, "b200mm_gqa_decode")
    return out


def apply_decode_attn(model: nn.Module) -> nn.Module:
    """Set ``decode_attn_op = b200_decode_attn`` on every layer's attention
    that has the hook (the engine ``Attention`` and this package's fused-QKV
    modules).  Returns ``model``."""
    for block in model.layers:
        if hasattr(block.attn, "decode_attn_op"):
            block.attn.decode_attn_op = b200_decode_attn
    return model
