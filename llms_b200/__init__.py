"""llms_b200: the B200-native (sm_100a) matmul hot path of the llms Qwen3 engine.

Subpackages / modules:
  kernels  -- fused QKV, fused gate-up-SiLU, int8 weight-only (reference
              ``src/kernels`` API)
  mla      -- absorbed latent-KV MLA decode backend (reference
              ``engine/mla.py`` T == 1 branch)
The compute lives in ``_lib/libb200mm.so`` (C ABI: ``include/b200mm.h``).
"""

__version__ = "0.1.0"
