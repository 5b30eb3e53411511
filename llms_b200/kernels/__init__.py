"""B200 (sm_100a) kernels behind the reference engine's ``kernels`` API.

Same exports as the reference package (``kernels/__init__.py:3-14``), plus
the int8 weight-only variants, the ``o`` / ``down`` projections and the GQA
decode attention op.
"""

from .decode_attn import apply_decode_attn, b200_decode_attn
from .fused_ffn import TritonFFN, triton_fused_gate_up_silu
from .fused_qkv import TritonAttention, triton_fused_qkv
from .linear import B200Linear, Int8Linear, b200_linear, int8_linear
from .quant import (
    Int8Attention,
    Int8FFN,
    dequantize_per_row,
    int8_fused_gate_up_silu,
    int8_fused_qkv,
    quantize_per_row,
)
from .swap import apply_int8_kernels, apply_linear_kernels, apply_triton_kernels, prewarm_triton_kernels

__all__ = [
    "apply_decode_attn",
    "b200_decode_attn",
    "B200Linear",
    "Int8Linear",
    "apply_linear_kernels",
    "b200_linear",
    "int8_linear",
    "Int8Attention",
    "Int8FFN",
    "TritonAttention",
    "TritonFFN",
    "apply_int8_kernels",
    "apply_triton_kernels",
    "dequantize_per_row",
    "int8_fused_gate_up_silu",
    "int8_fused_qkv",
    "prewarm_triton_kernels",
    "quantize_per_row",
    "triton_fused_gate_up_silu",
    "triton_fused_qkv",
]
