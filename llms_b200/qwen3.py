"""Qwen3-shaped decoder around the B200 projections (caller of the hot path).

The reference engine's model (engine/model.py:27-185) restated just far
enough to run a decode step: embedding, decoder blocks (pre-norm GQA
attention with QK-norm and RoPE, SwiGLU FFN), final norm, LM head, and the
contiguous KV cache of engine/kv_cache.py.  Module and parameter names match
the reference, so `apply_triton_kernels` / `apply_int8_kernels` swap the same
attributes they swap in the reference engine.

`synthetic_int8_model` builds BASELINE config 5 directly in int8
(per-output-row scales), without materialising a bf16 copy of the fused
projections, and `Qwen3Model.forward_fp32_dequant` is the fp32 check path:
the same model run eagerly in fp32 with every int8 weight dequantised, one
layer at a time, TF32 disabled.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .kernels._eager import RMSNorm, rope
from .kernels.fused_qkv import _one_buffer
from .kernels.glue import fits_qk_norm_rope, fits_rms_norm, qk_norm_rope_cache, rms_norm
from .kernels.quant import Int8Attention, Int8FFN, dequantize_per_row


@dataclass(frozen=True)
class Qwen3Shape:
    vocab_size: int = 151936
    hidden_size: int = 4096
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 12288
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 4096


QWEN3_8B = Qwen3Shape()
QWEN3_4B = Qwen3Shape(hidden_size=2560, intermediate_size=9728)


@dataclass
class KVCache:
    """Per-layer (max_batch, num_kv_heads, max_seq_len, head_dim) K and V."""

    k: list
    v: list
    cur_len: int = 0

    @classmethod
    def alloc(cls, *, num_layers, max_batch, num_kv_heads, max_seq_len, head_dim, dtype, device) -> "KVCache":
        shape = (max_batch, num_kv_heads, max_seq_len, head_dim)
        return cls(k=[torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)],
                   v=[torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)])


def rope_tables(head_dim: int, max_pos: int, theta: float, device=None):
    """cos/sin (max_pos, head_dim), concat convention (engine/attention.py:36-55)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    emb = torch.cat([ang, ang], dim=-1)
    return emb.cos().to(device), emb.sin().to(device)


def attention_core(q, k, v, kv_cache, layer_idx, start_pos, n_rep, decode_op=None):
    """Cache write + GQA SDPA of engine/attention.py:122-149 (q, k, v: B, H, T, D);
    a single-query step goes to ``decode_op`` when one is set (:138-145)."""
    B, _, T, _ = q.shape
    end = start_pos + T
    kv_cache.k[layer_idx][:B, :, start_pos:end] = k
    kv_cache.v[layer_idx][:B, :, start_pos:end] = v
    fk = kv_cache.k[layer_idx][:B, :, :end]
    fv = kv_cache.v[layer_idx][:B, :, :end]
    if T == 1 and decode_op is not None:
        return decode_op(q, fk, fv, scale=q.shape[-1] ** -0.5, layer_idx=layer_idx)
    if n_rep > 1:
        fk = fk.repeat_interleave(n_rep, dim=1)
        fv = fv.repeat_interleave(n_rep, dim=1)
    if T == 1:
        return F.scaled_dot_product_attention(q, fk, fv, is_causal=False)
    qp = torch.arange(start_pos, end, device=q.device).unsqueeze(1)
    kp = torch.arange(0, end, device=q.device).unsqueeze(0)
    return F.scaled_dot_product_attention(q, fk, fv, attn_mask=qp >= kp)


def _project_qkv(attn, x):
    """q, k, v of any attention module here (the engine's q/k/v Linears, or the
    fused / int8 / sharded modules' ``project_qkv``)."""
    if hasattr(attn, "project_qkv"):
        return attn.project_qkv(x)
    return attn.q(x), attn.k(x), attn.v(x)


def static_decode_attention(attn, x, kv_cache, layer_idx, cos, sin, pos, tables=None):
    """One decode token (x: B, 1, C) through ``attn`` with its position ``pos``
    a device tensor: the cache row is written with ``index_copy_`` and the
    softmax runs over the whole static cache with a mask computed on the
    device, so nothing in it depends on a host-side position (what a CUDA graph
    replayed at every position needs).  Same result as the engine's T == 1
    path (engine/attention.py:119-163).

    Two limits of this static form: the softmax reads the cache's whole
    capacity (``max_seq_len`` rows, masked) at every position, so a step
    costs time for the capacity, not the current length; and
    ``attn.decode_attn_op`` is not used here (the GQA decode kernel takes the
    length on the host), so a captured step runs torch's SDPA."""
    B = x.shape[0]
    H, KV, D = attn.num_heads, attn.num_kv_heads, attn.head_dim
    qf, kf, vf = _project_qkv(attn, x)
    kc, vc = kv_cache.k[layer_idx][:B], kv_cache.v[layer_idx][:B]
    flat = _one_buffer(qf, kf, vf)
    if (tables is not None and flat is not None and kc.dtype == flat.dtype
            and fits_qk_norm_rope(flat, attn.q_norm, attn.k_norm, tables[0], D)):
        # norms, RoPE (position read on the device) and the cache write in one launch
        q = qk_norm_rope_cache(flat, attn.q_norm, attn.k_norm, tables[0], tables[1], num_heads=H, num_kv_heads=KV,
                               head_dim=D, k_cache=kc, v_cache=vc, pos=pos)
    else:
        q = attn.q_norm(qf.reshape(B, 1, H, D)).transpose(1, 2)
        k = attn.k_norm(kf.reshape(B, 1, KV, D)).transpose(1, 2)
        v = vf.reshape(B, 1, KV, D).transpose(1, 2)
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        kc.index_copy_(2, pos, k.to(kc.dtype))
        vc.index_copy_(2, pos, v.to(vc.dtype))
    S = kc.shape[2]
    mask = (torch.arange(S, device=x.device) <= pos).view(1, 1, 1, S)
    a = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, enable_gqa=H != KV)
    return attn.o(a.transpose(1, 2).reshape(B, 1, H * D))


class Attention(nn.Module):
    """Eager GQA attention with QK-norm and RoPE (engine/attention.py:79-163)."""

    def __init__(self, shape: Qwen3Shape) -> None:
        super().__init__()
        H, KV, D, C = shape.num_attention_heads, shape.num_key_value_heads, shape.head_dim, shape.hidden_size
        self.num_heads, self.num_kv_heads, self.head_dim = H, KV, D
        self.q = nn.Linear(C, H * D, bias=False)
        self.k = nn.Linear(C, KV * D, bias=False)
        self.v = nn.Linear(C, KV * D, bias=False)
        self.o = nn.Linear(H * D, C, bias=False)
        self.q_norm = RMSNorm(D, shape.rms_norm_eps)
        self.k_norm = RMSNorm(D, shape.rms_norm_eps)
        self.decode_attn_op = None  # engine/attention.py:101-105

    def forward(self, x, *, kv_cache, layer_idx, cos, sin, start_pos):
        B, T, _ = x.shape
        q = self.q_norm(self.q(x).view(B, T, self.num_heads, self.head_dim)).transpose(1, 2)
        k = self.k_norm(self.k(x).view(B, T, self.num_kv_heads, self.head_dim)).transpose(1, 2)
        v = self.v(x).view(B, T, self.num_kv_heads, self.head_dim).transpose(1, 2)
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        a = attention_core(q, k, v, kv_cache, layer_idx, start_pos, self.num_heads // self.num_kv_heads,
                           self.decode_attn_op)
        return self.o(a.transpose(1, 2).reshape(B, T, self.num_heads * self.head_dim))


class FFN(nn.Module):
    """SwiGLU: down(silu(gate(x)) * up(x)) (engine/model.py:27-37)."""

    def __init__(self, hidden: int, inter: int) -> None:
        super().__init__()
        self.gate = nn.Linear(hidden, inter, bias=False)
        self.up = nn.Linear(hidden, inter, bias=False)
        self.down = nn.Linear(inter, hidden, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class DecoderBlock(nn.Module):
    def __init__(self, shape: Qwen3Shape, *, build_projections: bool = True) -> None:
        super().__init__()
        self.norm1 = RMSNorm(shape.hidden_size, shape.rms_norm_eps)
        self.norm2 = RMSNorm(shape.hidden_size, shape.rms_norm_eps)
        if build_projections:
            self.attn = Attention(shape)
            self.ffn = FFN(shape.hidden_size, shape.intermediate_size)

    def forward(self, x, *, kv_cache, layer_idx, cos, sin, start_pos):
        h = x + self.attn(self.norm1(x), kv_cache=kv_cache, layer_idx=layer_idx, cos=cos, sin=sin,
                          start_pos=start_pos)
        return h + self.ffn(self.norm2(h))


class Qwen3Model(nn.Module):
    """engine/model.py:76-185 (untied LM head)."""

    def __init__(self, shape: Qwen3Shape, *, build_projections: bool = True) -> None:
        super().__init__()
        self.shape = shape
        self.embed = nn.Embedding(shape.vocab_size, shape.hidden_size)
        self.layers = nn.ModuleList(
            [DecoderBlock(shape, build_projections=build_projections) for _ in range(shape.num_hidden_layers)])
        self.final_norm = RMSNorm(shape.hidden_size, shape.rms_norm_eps)
        self.lm_head = nn.Linear(shape.hidden_size, shape.vocab_size, bias=False)
        cos, sin = rope_tables(shape.head_dim, shape.max_position_embeddings, shape.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def forward(self, input_ids, kv_cache, start_pos=None):
        if start_pos is None:
            start_pos = kv_cache.cur_len
        T = input_ids.shape[1]
        h = self.embed(input_ids)
        cos = self.rope_cos[start_pos:start_pos + T].to(h.dtype)
        sin = self.rope_sin[start_pos:start_pos + T].to(h.dtype)
        if self._fused_norms_fit(h):
            y = self._blocks_fused(h, lambda blk, i, x: blk.attn(x, kv_cache=kv_cache, layer_idx=i, cos=cos,
                                                                 sin=sin, start_pos=start_pos))
        else:
            for i, layer in enumerate(self.layers):
                h = layer(h, kv_cache=kv_cache, layer_idx=i, cos=cos, sin=sin, start_pos=start_pos)
            y = self.final_norm(h)
        logits = self.lm_head(y)
        kv_cache.cur_len = start_pos + T
        return logits

    def _fused_norms_fit(self, h: torch.Tensor) -> bool:
        if not getattr(self, "fused_glue", True):
            return False
        norms = [self.final_norm] + [n for blk in self.layers for n in (blk.norm1, blk.norm2)]
        return all(fits_rms_norm(h, n.weight) for n in norms)

    def _blocks_fused(self, h: torch.Tensor, attn):
        """The decoder blocks with every norm and residual add on
        ``b200mm_rmsnorm``: block i computes h = x + attn(norm1(x)) and
        x' = h + ffn(norm2(h)) (engine/model.py:54-63); each residual add is
        folded into the norm that reads its result, so a block is two norm
        launches around its attention and FFN, and the last add is folded
        into the final norm.  Returns final_norm(x_last)."""
        x, f = h, None
        for i, blk in enumerate(self.layers):
            if f is None:
                y = rms_norm(x, blk.norm1.weight, blk.norm1.eps)
            else:
                x, y = rms_norm(f, blk.norm1.weight, blk.norm1.eps, residual=x)
            a = attn(blk, i, y)
            x, y = rms_norm(a, blk.norm2.weight, blk.norm2.eps, residual=x)
            f = blk.ffn(y)
        _, y = rms_norm(f, self.final_norm.weight, self.final_norm.eps, residual=x)
        return y

    def forward_static(self, input_ids: torch.Tensor, kv_cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        """One decode step (input_ids: B, 1) at the position held in the device
        tensor ``pos`` (shape (1,), int64): the same blocks as ``forward``, with
        the RoPE rows picked and the cache written on the device
        (``static_decode_attention``), so one captured CUDA graph serves every
        position.  Does not touch ``kv_cache.cur_len``."""
        h = self.embed(input_ids)
        cos = self.rope_cos.index_select(0, pos).to(h.dtype)
        sin = self.rope_sin.index_select(0, pos).to(h.dtype)
        if self._fused_norms_fit(h):
            return self.lm_head(self._blocks_fused(
                h, lambda blk, i, x: static_decode_attention(blk.attn, x, kv_cache, i, cos, sin, pos,
                                                             tables=(self.rope_cos, self.rope_sin))))
        for i, blk in enumerate(self.layers):
            h = h + static_decode_attention(blk.attn, blk.norm1(h), kv_cache, i, cos, sin, pos)
            h = h + blk.ffn(blk.norm2(h))
        return self.lm_head(self.final_norm(h))

    def alloc_cache(self, max_seq_len, *, max_batch=1, dtype=None, device=None) -> KVCache:
        p = self.lm_head.weight
        return KVCache.alloc(num_layers=len(self.layers), max_batch=max_batch,
                             num_kv_heads=self.shape.num_key_value_heads, max_seq_len=max_seq_len,
                             head_dim=self.shape.head_dim, dtype=dtype or p.dtype, device=device or p.device)

    # ---- fp32 check path ----------------------------------------------------
    @torch.no_grad()
    def forward_fp32_dequant(self, input_ids, kv_cache, start_pos):
        """The same forward in fp32 eager torch, every int8 weight dequantised
        (W = q * s), one layer at a time; TF32 off.  `kv_cache` must be fp32."""
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            S = self.shape
            T = input_ids.shape[1]
            h = self.embed(input_ids).float()
            cos = self.rope_cos[start_pos:start_pos + T].float()
            sin = self.rope_sin[start_pos:start_pos + T].float()
            nq, nk = S.num_attention_heads * S.head_dim, S.num_key_value_heads * S.head_dim
            for i, blk in enumerate(self.layers):
                a, f = blk.attn, blk.ffn
                B = h.shape[0]
                x = blk.norm1(h)
                W = dequantize_per_row(a.q_qkv, a.s_qkv)
                y = x @ W.T
                del W
                q = y[..., :nq].view(B, T, S.num_attention_heads, S.head_dim)
                k = y[..., nq:nq + nk].view(B, T, S.num_key_value_heads, S.head_dim)
                v = y[..., nq + nk:].view(B, T, S.num_key_value_heads, S.head_dim)
                q = a.q_norm(q).float().transpose(1, 2)
                k = a.k_norm(k).float().transpose(1, 2)
                v = v.transpose(1, 2)
                q, k = rope(q, cos, sin), rope(k, cos, sin)
                att = attention_core(q, k, v, kv_cache, i, start_pos, S.num_attention_heads // S.num_key_value_heads)
                h = h + att.transpose(1, 2).reshape(B, T, nq) @ a.o.weight.float().T
                x = blk.norm2(h)
                g = x @ dequantize_per_row(f.qg, f.sg).T
                u = x @ dequantize_per_row(f.qu, f.su).T
                h = h + (F.silu(g) * u) @ f.down.weight.float().T
            return self.final_norm(h) @ self.lm_head.weight.float().T
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev


class GraphedDecodeStep:
    """A whole decode step of ``model`` (every layer, the LM head) captured once
    as a CUDA graph and replayed at every position: the token ids and the
    position are copied into static device buffers, then one graph launch
    replaces the step's hundreds of kernel launches from Python (the dispatch
    overhead the engine's own profiling names as the end-to-end blocker,
    bench/profile.py:412-420).

    ``step = GraphedDecodeStep(model, cache, batch)`` after the prefill;
    ``logits = step(ids, pos)`` for each new token (ids: (batch, 1) on the
    device).  The returned logits live in a static buffer overwritten by the
    next call.  Building the graph runs the step once at ``cache.cur_len``,
    the row the first real step writes anyway."""

    def __init__(self, model: Qwen3Model, kv_cache: KVCache, batch: int) -> None:
        dev = model.lm_head.weight.device
        self.model, self.cache = model, kv_cache
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.pos = torch.full((1,), kv_cache.cur_len, dtype=torch.long, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s), torch.inference_mode():  # first-call set-up outside the capture
            model.forward_static(self.ids, kv_cache, self.pos)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.inference_mode():
            self.logits = model.forward_static(self.ids, kv_cache, self.pos)

    def __call__(self, ids: torch.Tensor, pos: int) -> torch.Tensor:
        S = self.cache.k[0].shape[2]
        if not 0 <= pos < S:
            raise ValueError(f"position {pos} is outside the cache (rows 0..{S - 1})")
        if tuple(ids.shape) != tuple(self.ids.shape):
            raise ValueError(f"ids shape {tuple(ids.shape)} != the captured step's {tuple(self.ids.shape)}")
        self.ids.copy_(ids)
        self.pos.fill_(pos)
        self.graph.replay()
        self.cache.cur_len = pos + 1
        return self.logits


def greedy(logits: torch.Tensor) -> torch.Tensor:
    """Argmax along the vocabulary (engine/sampler.py:17-19)."""
    return logits.argmax(dim=-1)


def _int8_block(shape: Qwen3Shape, device, dtype):
    """An empty decoder block of int8 fused QKV / gate-up modules (buffers
    ``q_qkv, s_qkv`` and ``qg, sg, qu, su``) with bf16 ``o`` / ``down``."""
    C, I = shape.hidden_size, shape.intermediate_size
    H, KV, D = shape.num_attention_heads, shape.num_key_value_heads, shape.head_dim
    att = Int8Attention.__new__(Int8Attention)
    nn.Module.__init__(att)
    att.hidden_size, att.num_heads, att.num_kv_heads, att.head_dim = C, H, KV, D
    att.n_q, att.n_k = H * D, KV * D
    att.register_buffer("q_qkv", torch.empty(H * D + 2 * KV * D, C, device=device, dtype=torch.int8))
    att.register_buffer("s_qkv", torch.empty(H * D + 2 * KV * D, device=device))
    att.o = nn.Linear(H * D, C, bias=False, device=device, dtype=dtype)
    att.q_norm = RMSNorm(D, shape.rms_norm_eps).to(device=device, dtype=dtype)
    att.k_norm = RMSNorm(D, shape.rms_norm_eps).to(device=device, dtype=dtype)
    att.decode_attn_op = None
    ffn = Int8FFN.__new__(Int8FFN)
    nn.Module.__init__(ffn)
    for name in ("g", "u"):
        ffn.register_buffer("q" + name, torch.empty(I, C, device=device, dtype=torch.int8))
        ffn.register_buffer("s" + name, torch.empty(I, device=device))
    ffn.down = nn.Linear(I, C, bias=False, device=device, dtype=dtype)
    return att, ffn


def _int8_skeleton(shape: Qwen3Shape, device, dtype) -> Qwen3Model:
    m = Qwen3Model(shape, build_projections=False)
    m.to(device=device, dtype=dtype)
    for blk in m.layers:
        blk.attn, blk.ffn = _int8_block(shape, device, dtype)
    return m


@torch.no_grad()
def int8_model_from_state(state: dict, shape: Qwen3Shape, *, device="cuda", dtype=torch.bfloat16) -> Qwen3Model:
    """A model of int8 fused QKV / gate-up blocks loaded from ``state``
    (tensors or numpy arrays named as ``oracle.inputs.cfg5_model`` writes
    them: ``layers.i.attn.q_qkv`` / ``s_qkv``, ``layers.i.ffn.qg`` / ``sg`` /
    ``qu`` / ``su``, the dense ``embed``, ``attn.o``, ``ffn.down`` and
    ``lm_head`` weights, optional norm weights).  Every parameter and buffer
    of the model must be covered, except norm weights (default one)."""
    m = _int8_skeleton(shape, device, dtype)
    own = dict(m.named_parameters())
    own.update(dict(m.named_buffers()))
    own = {k: v for k, v in own.items() if not k.startswith("rope_")}
    missing = [k for k in own if k not in state and "norm" not in k]
    unknown = [k for k in state if k not in own]
    if missing or unknown:
        raise ValueError(f"state mismatch: missing={missing[:8]}, unexpected={unknown[:8]}")
    for k, v in state.items():
        t = torch.as_tensor(v)
        own[k].copy_(t.to(own[k].dtype) if t.dtype != own[k].dtype else t)
    return m.eval()


@torch.no_grad()
def dequantized_dense_model(model: Qwen3Model) -> Qwen3Model:
    """The reference engine's arithmetic for an int8 model: every int8 fused
    projection dequantised (``W = q * s``), rounded to the model dtype and
    split back into the engine's q / k / v and gate / up ``nn.Linear``s
    (engine/attention.py:95-98, engine/model.py:30-32); ``o``, ``down``,
    norms, embedding and LM head shared with ``model``; norms and residual
    adds as the engine's eager torch ops (``fused_glue = False``)."""
    shape, p = model.shape, model.lm_head.weight
    out = Qwen3Model(shape, build_projections=False)
    out.to(device=p.device, dtype=p.dtype)
    out.fused_glue = False  # the engine's own eager norms and adds, too
    out.embed, out.lm_head, out.final_norm = model.embed, model.lm_head, model.final_norm
    nq = shape.num_attention_heads * shape.head_dim
    nk = shape.num_key_value_heads * shape.head_dim
    for src, dst in zip(model.layers, out.layers):
        a, f = src.attn, src.ffn
        att = Attention.__new__(Attention)
        nn.Module.__init__(att)
        att.num_heads, att.num_kv_heads, att.head_dim = a.num_heads, a.num_kv_heads, a.head_dim
        W = dequantize_per_row(a.q_qkv, a.s_qkv).to(p.dtype)
        for name, w in zip(("q", "k", "v"), W.split([nq, nk, nk])):
            setattr(att, name, nn.Linear(w.shape[1], w.shape[0], bias=False, device=p.device, dtype=p.dtype))
            getattr(att, name).weight.copy_(w)
        del W
        att.o, att.q_norm, att.k_norm, att.decode_attn_op = a.o, a.q_norm, a.k_norm, None
        ffn = FFN.__new__(FFN)
        nn.Module.__init__(ffn)
        for name, (q, s) in (("gate", (f.qg, f.sg)), ("up", (f.qu, f.su))):
            w = dequantize_per_row(q, s).to(p.dtype)
            setattr(ffn, name, nn.Linear(w.shape[1], w.shape[0], bias=False, device=p.device, dtype=p.dtype))
            getattr(ffn, name).weight.copy_(w)
            del w
        ffn.down = f.down
        dst.norm1, dst.norm2 = src.norm1, src.norm2
        dst.attn, dst.ffn = att, ffn
    return out.eval()


@torch.no_grad()
def synthetic_int8_model(shape: Qwen3Shape = QWEN3_8B, *, seed: int = 4, device="cuda",
                         dtype=torch.bfloat16) -> Qwen3Model:
    """fused QKV and gate/up weights int8 ~ U{-127..127}
    with per-output-row scales ~ U(1e-4, 1e-3); everything else (embedding,
    o, down, LM head) bf16 ~ N(0, 0.02), norms 1.  Seeded on `device`."""
    g = torch.Generator(device=device).manual_seed(seed)
    m = _int8_skeleton(shape, device, dtype)

    def normal_(t):
        t.copy_(torch.randn(t.shape, generator=g, device=device, dtype=torch.float32) * 0.02)

    def int8_(q, s):
        q.copy_(torch.randint(-127, 128, q.shape, generator=g, device=device, dtype=torch.int8))
        s.copy_(torch.rand(s.shape, generator=g, device=device) * 9e-4 + 1e-4)

    normal_(m.embed.weight)
    normal_(m.lm_head.weight)
    for blk in m.layers:
        att, ffn = blk.attn, blk.ffn
        int8_(att.q_qkv, att.s_qkv)
        normal_(att.o.weight)
        int8_(ffn.qg, ffn.sg)
        int8_(ffn.qu, ffn.su)
        normal_(ffn.down.weight)
    return m.eval()
