"""In-place swap of engine modules for their B200-kernel counterparts.

Mirrors ``kernels/swap.py`` of the reference (``apply_triton_kernels``
lines 22-46, ``prewarm_triton_kernels`` lines 49-111) and adds the int8
weight-only swap.  The engine files stay untouched: the walker replaces
``block.ffn`` / ``block.attn`` on every ``model.layers`` entry.
"""

from __future__ import annotations

import torch
from torch import nn

from .fused_ffn import TritonFFN
from .fused_qkv import TritonAttention, triton_fused_qkv
from .linear import B200Linear, Int8Linear
from .quant import Int8Attention, Int8FFN, int8_fused_qkv


def apply_triton_kernels(model: nn.Module, *, fused_ffn: bool = True, fused_qkv: bool = True) -> nn.Module:
    """Replace each layer's ``ffn`` with :class:`TritonFFN` and ``attn`` with
    :class:`TritonAttention` (idempotent; returns ``model``)."""
    for block in model.layers:
        if fused_ffn and not isinstance(block.ffn, (TritonFFN, Int8FFN)):
            block.ffn = TritonFFN.from_eager(block.ffn)
        if fused_qkv and not isinstance(block.attn, TritonAttention) and hasattr(block.attn, "v"):
            block.attn = TritonAttention.from_eager(block.attn)
    return model


def apply_int8_kernels(model: nn.Module, *, ffn: bool = True, qkv: bool = True) -> nn.Module:
    """Quantise each layer's gate/up and q/k/v weights to int8 per output row
    and swap in :class:`Int8FFN` / :class:`Int8Attention` (idempotent)."""
    for block in model.layers:
        if ffn and not isinstance(block.ffn, Int8FFN):
            block.ffn = Int8FFN.from_eager(block.ffn)
        if qkv and not isinstance(block.attn, Int8Attention) and (
            hasattr(block.attn, "v") or hasattr(block.attn, "W_qkv")
        ):
            block.attn = Int8Attention.from_eager(block.attn)
    return model


def apply_linear_kernels(model: nn.Module, *, int8: bool = False, o: bool = True, down: bool = True,
                         lm_head: bool = False) -> nn.Module:
    """Route each layer's attention output projection ``attn.o`` and FFN
    ``ffn.down`` through the B200 projection kernels (:class:`B200Linear`,
    sharing the weight; or :class:`Int8Linear` with ``int8=True``).  Works on
    the engine modules and on the fused-kernel modules alike, since both call
    ``self.o(...)`` / ``self.down(...)``.  ``lm_head=True`` routes the
    model's untied LM head (engine/model.py:93-96) the same way.  Idempotent;
    returns ``model``."""
    cls = Int8Linear if int8 else B200Linear
    for block in model.layers:
        if o and isinstance(block.attn.o, nn.Linear):
            block.attn.o = cls.from_linear(block.attn.o)
        if down and isinstance(block.ffn.down, nn.Linear):
            block.ffn.down = cls.from_linear(block.ffn.down)
    if lm_head and isinstance(getattr(model, "lm_head", None), nn.Linear):
        model.lm_head = cls.from_linear(model.lm_head)
    return model


def prewarm_triton_kernels(model: nn.Module, *, m_values: tuple[int, ...] = (1, 2, 3, 4, 5, 6, 7, 8)) -> None:
    """Run every swapped projection once per M in ``m_values`` (one module per
    distinct weight shape), so first-call costs (kernel attribute setup,
    occupancy queries) land outside timed regions.  The kernels have no
    autotuning, so this never changes later outputs."""
    ffns: dict[tuple, nn.Module] = {}
    attns: dict[tuple, nn.Module] = {}
    for m in model.modules():
        if isinstance(m, TritonFFN):
            ffns.setdefault(("d",) + tuple(m.gate.weight.shape), m)
        elif isinstance(m, Int8FFN):
            ffns.setdefault(("q",) + tuple(m.qg.shape), m)
        elif isinstance(m, Int8Attention):
            attns.setdefault(("q",) + tuple(m.q_qkv.shape), m)
        elif isinstance(m, TritonAttention):
            attns.setdefault(("d",) + tuple(m.W_qkv.shape), m)
    if not ffns and not attns:
        return
    with torch.inference_mode():
        for key, ffn in ffns.items():
            K = key[2]
            if isinstance(ffn, TritonFFN):
                dev, dt = ffn.gate.weight.device, ffn.gate.weight.dtype
            else:
                dev, dt = ffn.qg.device, ffn.down.weight.dtype
            for M in m_values:
                ffn(torch.zeros((1, M, K), dtype=dt, device=dev))
        for key, attn in attns.items():
            K = key[2]
            for M in m_values:
                if isinstance(attn, Int8Attention):
                    x = torch.zeros((1, M, K), dtype=attn.o.weight.dtype, device=attn.q_qkv.device)
                    int8_fused_qkv(x, attn.q_qkv, attn.s_qkv, n_q=attn.n_q, n_k=attn.n_k)
                else:
                    x = torch.zeros((1, M, K), dtype=attn.W_qkv.dtype, device=attn.W_qkv.device)
                    triton_fused_qkv(x, attn.W_qkv, n_q=attn.n_q, n_k=attn.n_k)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
