"""Seeded synthetic inputs for the BASELINE configurations.

TEST INFRASTRUCTURE ONLY for the checker side; ``bench.py`` and the GPU
tests use the same generators so the GPU and the oracle see identical
values.  Generator: numpy PCG64 (stable across numpy versions), float32
draws, rounded to bf16-representable values where the config is bf16 (the
arrays stay float32 so numpy can hold them).
"""

from __future__ import annotations

import numpy as np

QWEN3_4B = dict(hidden=2560, n_q=4096, n_k=1024, inter=9728)
QWEN3_8B = dict(hidden=4096, n_q=4096, n_k=1024, inter=12288, layers=36)
MLA_4B = dict(H=32, KV=8, D=128, DR=32, R=256, theta=1e6, eps=1e-6)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 -> nearest-even bf16, returned as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _normal(rng, shape, std=1.0):
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)


def cfg1(seed: int = 0):
    """Qwen3-0.6B FFN shape, fp32: x [4,1024], Wg/Wu [3072,1024]."""
    rng = np.random.default_rng(seed)
    x = _normal(rng, (4, 1024))
    wg = _normal(rng, (3072, 1024), 0.02)
    wu = _normal(rng, (3072, 1024), 0.02)
    return x, wg, wu


def cfg2(M: int, seed: int = 1, K: int = 2560, n_q: int = 4096, n_k: int = 1024):
    """Qwen3-4B fused QKV, bf16: x [M,K], W_qkv [n_q+2n_k, K]."""
    rng = np.random.default_rng(seed)
    x = round_bf16(_normal(rng, (M, K)))
    w = round_bf16(_normal(rng, (n_q + 2 * n_k, K), 0.02))
    return x, w


def cfg3(M: int, seed: int = 2, K: int = 2560, N: int = 9728):
    """Qwen3-4B gate-up, bf16: x [M,K], Wg||Wu [2N,K] -> (x, Wg, Wu)."""
    rng = np.random.default_rng(seed)
    x = round_bf16(_normal(rng, (M, K)))
    w = round_bf16(_normal(rng, (2 * N, K), 0.02))
    return x, w[:N], w[N:]


def o_down(M: int, which: str, seed: int = 6, hidden: int = 2560, n_q: int = 4096, inter: int = 9728):
    """Qwen3-4B output projection (``which="o"``: W [hidden, n_q]) or down
    projection (``"down"``: W [hidden, inter]), bf16 -> (x, W)."""
    K = n_q if which == "o" else inter
    rng = np.random.default_rng(seed + (0 if which == "o" else 1))
    x = round_bf16(_normal(rng, (M, K)))
    w = round_bf16(_normal(rng, (hidden, K), 0.02))
    return x, w


def cfg4(B: int, L: int, seed: int = 3, H=32, KV=8, D=128, DR=32, R=256):
    """MLA latent decode, bf16: c_kv [B,L,R], kr [B,L,KV,DR], W_UK [KV,D-DR,R],
    W_UV [KV,D,R] (std 1/4, i.e. variance 1/16), q [B,H,D]; k_norm weight ones."""
    rng = np.random.default_rng(seed)
    c = round_bf16(_normal(rng, (B, L, R)))
    kr = round_bf16(_normal(rng, (B, L, KV, DR)))
    w_uk = round_bf16(_normal(rng, (KV, D - DR, R), 0.25))
    w_uv = round_bf16(_normal(rng, (KV, D, R), 0.25))
    q = round_bf16(_normal(rng, (B, H, D)))
    k_norm_w = np.ones(D, np.float32)
    return dict(q=q, c_kv=c, k_rope_pre=kr, w_uk=w_uk, w_uv=w_uv, k_norm_w=k_norm_w)


def int8_weight(rng, N: int, K: int):
    """int8 ~ U{-127..127}, scales ~ U(1e-4, 1e-3) fp32 (config 5)."""
    q = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = rng.uniform(1e-4, 1e-3, size=(N,)).astype(np.float32)
    return q, s


def cfg5_layer(seed: int = 4, M: int = 1, K: int = 4096, n_q=4096, n_k=1024, inter=12288):
    """One Qwen3-8B layer's int8 projections + a bf16 activation batch."""
    rng = np.random.default_rng(seed)
    x = round_bf16(_normal(rng, (M, K)))
    qkv_q, qkv_s = int8_weight(rng, n_q + 2 * n_k, K)
    gu_q, gu_s = int8_weight(rng, 2 * inter, K)
    return dict(x=x, qkv_q=qkv_q, qkv_s=qkv_s, gate_q=gu_q[:inter], gate_s=gu_s[:inter],
                up_q=gu_q[inter:], up_s=gu_s[inter:])


def cfg5_model(layers: int = 2, vocab: int = 4096, seed: int = 4, hidden: int = 4096, n_q: int = 4096,
               n_k: int = 1024, inter: int = 12288):
    """Weights of a Qwen3-8B-shaped model (config 5) with ``layers`` decoder
    blocks and a ``vocab``-row embedding / LM head, as a state dict of numpy
    arrays named like the engine's modules (engine/model.py:40-106): int8
    fused QKV ``layers.i.attn.q_qkv`` [n_q + 2 n_k, hidden] and gate / up
    ``layers.i.ffn.qg`` / ``qu`` [inter, hidden] with fp32 per-row scales
    (``s_qkv``, ``sg``, ``su``); bf16-representable N(0, 0.02) ``embed``,
    ``attn.o``, ``ffn.down`` and ``lm_head``; RMSNorm weights one."""
    rng = np.random.default_rng(seed)
    st = {"embed.weight": round_bf16(_normal(rng, (vocab, hidden), 0.02))}
    for i in range(layers):
        p = f"layers.{i}."
        st[p + "attn.q_qkv"], st[p + "attn.s_qkv"] = int8_weight(rng, n_q + 2 * n_k, hidden)
        st[p + "attn.o.weight"] = round_bf16(_normal(rng, (hidden, n_q), 0.02))
        st[p + "ffn.qg"], st[p + "ffn.sg"] = int8_weight(rng, inter, hidden)
        st[p + "ffn.qu"], st[p + "ffn.su"] = int8_weight(rng, inter, hidden)
        st[p + "ffn.down.weight"] = round_bf16(_normal(rng, (hidden, inter), 0.02))
    st["lm_head.weight"] = round_bf16(_normal(rng, (vocab, hidden), 0.02))
    return st


def cfg5_tokens(batch: int, prompt: int, vocab: int, seed: int = 104):
    """Prompt ids [batch, prompt] and the next token ids [batch, 1]."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, size=(batch, prompt + 1), dtype=np.int64)
    return ids[:, :prompt], ids[:, prompt:]


def mla_module(hidden: int = 2560, seed: int = 9, H=32, KV=8, D=128, DR=32, R=256):
    """Weights of one latent-attention layer at the Qwen3-4B MLA point, named
    as the reference ``MLAttention``'s state dict (engine/mla.py:134-150):
    projections N(0, 0.02) except ``uk_nope`` / ``uv`` N(0, 1/16) (std 1/4),
    ``q_norm`` one, ``k_norm`` 1 + N(0, 0.1); bf16-representable."""
    rng = np.random.default_rng(seed)
    w = lambda n, k, std: round_bf16(_normal(rng, (n, k), std))
    st = {"q.weight": w(H * D, hidden, 0.02), "dkv.weight": w(R, hidden, 0.02),
          "uk_nope.weight": w(KV * (D - DR), R, 0.25), "uv.weight": w(KV * D, R, 0.25),
          "kr.weight": w(KV * DR, hidden, 0.02), "o.weight": w(hidden, H * D, 0.02),
          "q_norm.weight": np.ones(D, np.float32),
          "k_norm.weight": round_bf16(1.0 + _normal(rng, (D,), 0.1))}
    return st


def mla_steps(B: int = 2, prefill: int = 20, decode: int = 3, hidden: int = 2560, seed: int = 10):
    """Layer inputs: a prefill block [B, prefill, hidden] then ``decode``
    single-token inputs [decode, B, 1, hidden], N(0, 1), bf16-representable."""
    rng = np.random.default_rng(seed)
    return round_bf16(_normal(rng, (B, prefill, hidden))), round_bf16(_normal(rng, (decode, B, 1, hidden)))
