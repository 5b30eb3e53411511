"""llms_b200: the B200-native (sm_100a) matmul hot path of the llms Qwen3 engine.

Subpackages / modules:
  kernels  -- fused QKV, fused gate-up-SiLU, int8 weight-only (reference
              ``src/kernels`` API), the ``o`` / ``down`` projections and the
              GQA decode attention op for the engine's ``decode_attn_op`` seam
  mla      -- absorbed latent-KV MLA decode backend (reference
              ``engine/mla.py`` T == 1 branch), with the fused "Q + latent"
              projection of the decode step
  qwen3    -- a Qwen3-shaped decoder around these ops (the caller of the path)
  shard    -- that decoder's decode step column-sharded over GPUs
The compute lives in ``_lib/libb200mm.so`` (C ABI: ``include/b200mm.h``).
"""

__version__ = "0.2.0"
