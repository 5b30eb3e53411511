"""Float64 numpy restatement of the reference engine's hot-path math.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Each function cites
the reference lines (paths inside the aaholmes/llms project) it restates.
Inputs are numpy arrays; computation is float64 unless stated.
"""

from __future__ import annotations

import numpy as np


def silu(g: np.ndarray) -> np.ndarray:
    # torch.nn.functional.silu(g) = g * sigmoid(g)
    return g / (1.0 + np.exp(-g))


def gate_up_silu(x: np.ndarray, wg: np.ndarray, wu: np.ndarray) -> np.ndarray:
    """``silu(x Wg^T) * (x Wu^T)`` -- engine/model.py:36-37 minus ``down``;
    contract tests/test_kernels_fused_ffn.py:21-30.  x: (..., K); W: (N, K)."""
    x = np.asarray(x, np.float64)
    return silu(x @ np.asarray(wg, np.float64).T) * (x @ np.asarray(wu, np.float64).T)


def qkv(x: np.ndarray, w_qkv: np.ndarray, n_q: int, n_k: int):
    """Row-stacked projection then split -- engine/attention.py:119-121;
    contract tests/test_kernels_fused_qkv.py:22-34; split as
    kernels/fused_qkv.py:147-148."""
    y = np.asarray(x, np.float64) @ np.asarray(w_qkv, np.float64).T
    return y[..., :n_q], y[..., n_q:n_q + n_k], y[..., n_q + n_k:]


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Bias-free ``nn.Linear``: the attention output projection
    ``self.o(attn)`` (engine/attention.py:163) and the FFN down projection
    ``self.down(...)`` (engine/model.py:37).  x: (..., K); W: (N, K)."""
    return np.asarray(x, np.float64) @ np.asarray(w, np.float64).T


def dequant(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """int8 weight-only storage: W[n, k] = q[n, k] * s[n] (new path; the
    oracle is dequantise-then-reference)."""
    return q.astype(np.float64) * np.asarray(s, np.float64)[:, None]


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """engine/attention.py:28-33 in float64 (the fp32 module with no dtype
    round trip): w * x * rsqrt(mean(x^2) + eps)."""
    x = np.asarray(x, np.float64)
    return np.asarray(w, np.float64) * x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def mla_inv_freq(head_dim: int, d_rope: int, theta: float) -> np.ndarray:
    """engine/mla.py:158-163: the first d_rope/2 entries of the head_dim-sized
    RoPE frequency vector, computed in float32 as the reference does."""
    import torch  # the reference computes this with torch in fp32; match it bit for bit

    full = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    return full[: d_rope // 2].numpy().astype(np.float32)


def rope_cos_sin(positions: np.ndarray, inv_freq: np.ndarray):
    """engine/mla.py:164-168: angles t * inv_freq in float32 (torch.outer on
    fp32), concatenated [freqs, freqs]; cos/sin evaluated here in float64."""
    ang = np.outer(positions.astype(np.float32), inv_freq.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([ang, ang], axis=-1).astype(np.float64)
    return np.cos(emb), np.sin(emb)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """engine/attention.py:58-61."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def mla_decode(q, c_kv, k_rope_pre, w_uk, w_uv, k_norm_w, eps, inv_freq, L, scale=None):
    """Decode step of MLAttention, T == 1 -- engine/mla.py:206-264 (before ``o``).

    Args (numpy):
        q:          (B, H, D)       query after q_norm, before RoPE (mla.py:195-197)
        c_kv:       (B, >=L, R)     latent cache
        k_rope_pre: (B, >=L, KV, DR) un-normed, un-rotated rope keys
        w_uk:       (KV, DN, R)     uk_nope.weight.view(KV, DN, R)
        w_uv:       (KV, D, R)      uv.weight.view(KV, D, R)
        k_norm_w:   (D,)
        inv_freq:   (DR/2,) float32
        L:          context length; the query sits at position L-1
    Returns:
        (B, H, D) float64 -- the SDPA output of mla.py:262 as (B, H, D).
    """
    q = np.asarray(q, np.float64)
    B, H, D = q.shape
    KV, DN, R = w_uk.shape
    DR = D - DN
    rep = H // KV
    c = np.asarray(c_kv[:, :L], np.float64)                      # (B, L, R)
    v = np.einsum("blr,gdr->blgd", c, np.asarray(w_uv, np.float64))  # mla.py:209
    k_nope = np.einsum("blr,gnr->blgn", c, np.asarray(w_uk, np.float64))  # mla.py:213
    k = np.concatenate([k_nope, np.asarray(k_rope_pre[:, :L], np.float64)], axis=-1)  # mla.py:215
    k = rms_norm(k, k_norm_w, eps)                              # mla.py:221
    if DR > 0:                                                  # mla.py:226-248
        cq, sq = rope_cos_sin(np.array([L - 1]), inv_freq)
        ck, sk = rope_cos_sin(np.arange(L), inv_freq)
        qr = q[..., DN:]
        q = np.concatenate([q[..., :DN], qr * cq[0] + rotate_half(qr) * sq[0]], axis=-1)
        kr = k[..., DN:]                                        # (B, L, KV, DR)
        kr = kr * ck[None, :, None, :] + rotate_half(kr) * sk[None, :, None, :]
        k = np.concatenate([k[..., :DN], kr], axis=-1)
    k = np.repeat(k, rep, axis=2)                               # mla.py:254-257
    v = np.repeat(v, rep, axis=2)
    if scale is None:
        scale = D ** -0.5                                       # SDPA default scale
    s = np.einsum("bhd,blhd->bhl", q, k) * scale                # mla.py:259-262 (mask all-true)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhl,blhd->bhd", p, v)


def mla_kv_scales(c_kv, k_rope_pre, w_uk, eps, D):
    """Per-token, per-group factor of the k_norm RMSNorm (mla.py:212-221):
    rsqrt(mean over the full head of [W_uk c ; kr]^2 + eps).  (B, T, KV)."""
    c = np.asarray(c_kv, np.float64)
    k_nope = np.einsum("btr,gnr->btgn", c, np.asarray(w_uk, np.float64))
    ss = (k_nope ** 2).sum(-1)
    if k_rope_pre is not None and k_rope_pre.shape[-1] > 0:
        ss = ss + (np.asarray(k_rope_pre, np.float64) ** 2).sum(-1)
    return 1.0 / np.sqrt(ss / D + eps)


def mla_rope_keys(k_rope_pre, k_norm_w, inv_freq, t0=0):
    """The RoPE'd rope half of the normed K head divided by its k_norm factor
    (engine/mla.py:221-242 with the per-token scalar factored out):
    rope_t(w_k[DN:] * kr_t) for positions t0, t0+1, ...  (B, T, KV, DR)."""
    kr = np.asarray(k_rope_pre, np.float64)
    DR = kr.shape[-1]
    w = np.asarray(k_norm_w, np.float64)[-DR:]
    cos, sin = rope_cos_sin(np.arange(t0, t0 + kr.shape[1]), inv_freq)
    z = kr * w
    return z * cos[None, :, None, :] + rotate_half(z) * sin[None, :, None, :]


def gqa_decode(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """Single-query GQA attention as the engine's decode step computes it:
    K/V expanded over the g = H / KV heads of each group (repeat_interleave)
    and ``scaled_dot_product_attention`` with no mask (engine/attention.py:
    147-150; the decode seam at :138-145 receives the unexpanded K/V).
    q: [B, H, D]; k, v: [B, KV, L, D] -> [B, H, D]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, H, D = q.shape
    g = H // k.shape[1]
    out = np.empty((B, H, D))
    for b in range(B):
        for h in range(H):
            s = k[b, h // g] @ q[b, h] * scale
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ v[b, h // g]
    return out
