"""Column-sharded decode step across GPUs (one process per GPU).

The multi-GPU form of the Qwen3-8B-shaped int8 decode step: every
projection of a layer is split by output columns across the ranks and
followed by one NCCL all-gather, the only collective the path uses:

* fused QKV, head-aligned: rank r holds q heads [r H / N, (r + 1) H / N)
  and the same share of the k and v heads (rows of the stacked [Wq; Wk; Wv]),
  so every rank's block is whole heads;
* gate-up-SiLU by intermediate columns (the gate and up rows of the same
  columns stay together, so SiLU * up is local);
* ``o`` and ``down`` by hidden columns.

The attention core (QK-norm, RoPE, the KV cache, softmax), the norms, the
embedding and the LM head run replicated on every rank, on the gathered
activations, so each rank holds the whole KV cache and produces the whole
logits.  Row-parallel projections with an all-reduce are not used (the path
allows gathers only).  Every projection is one of this package's kernels on
the local shard: ``int8_linear`` / ``int8_fused_gate_up_silu`` for the int8
projections and ``b200_linear`` for ``o`` / ``down``.

With a ``peer.PeerGather`` context (``shard_decode_model(..., peer=ctx)``)
the gathers run over NVLink into a region of their own per call site instead
of an NCCL all-gather plus a permute: at decode batch 1 (int8) / up to 4
(16-bit) the projection kernel itself stores its outputs into every rank's
region (``b200mm_*_peer``: compute and gather in one kernel); at larger
batches the projection is followed by one ``b200mm_peer_gather`` launch;
beyond the context's row budget, NCCL.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from . import _capi
from .kernels.linear import b200_linear, int8_linear
from .kernels.quant import Int8Attention, Int8FFN, int8_fused_gate_up_silu


def even_range(n: int, rank: int, world: int) -> range:
    """Rank ``rank``'s block of ``n`` columns; ``n`` must split evenly (the
    all-gather moves equal blocks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in [0, {world})")
    if n % world:
        raise ValueError(f"{n} columns do not split evenly over {world} ranks")
    per = n // world
    return range(rank * per, (rank + 1) * per)


def qkv_rows(n_q: int, n_k: int, rank: int, world: int) -> list[int]:
    """Rows of the stacked [Wq; Wk; Wv] that rank ``rank`` holds, head-aligned
    when the head counts split evenly (callers check that)."""
    q = even_range(n_q, rank, world)
    k = even_range(n_k, rank, world)
    return list(q) + [n_q + i for i in k] + [n_q + n_k + i for i in k]


def gather_cols(y: torch.Tensor, world: int, group=None, site=None) -> torch.Tensor:
    """All-gather each rank's column block of ``y`` (..., c) into (..., world c),
    blocks in rank order (over peer memory when ``site`` fits ``y``)."""
    if world == 1:
        return y
    if site is not None and site.fits(y):
        return site.gather(y)
    lead, c = y.shape[:-1], y.shape[-1]
    y2 = y.reshape(-1, c).contiguous()
    out = torch.empty((world * y2.shape[0], c), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(out, y2, group=group)
    return out.view(world, y2.shape[0], c).permute(1, 0, 2).reshape(*lead, world * c)


def gather_qkv(y: torch.Tensor, cq: int, ck: int, world: int, group=None, site=None):
    """All-gather per-rank [q_r | k_r | v_r] blocks (widths cq, ck, ck) into the
    full q (world cq), k and v (world ck), each in head order (over peer
    memory when ``site`` fits ``y``: views of one [..., world (cq + 2 ck)]
    buffer)."""
    lead = y.shape[:-1]
    if world == 1:
        return y.split([cq, ck, ck], dim=-1)
    if site is not None and site.fits(y):
        return site.gather(y, (cq, ck, ck)).split([world * cq, world * ck, world * ck], dim=-1)
    y2 = y.reshape(-1, cq + 2 * ck).contiguous()
    out = torch.empty((world * y2.shape[0], cq + 2 * ck), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(out, y2, group=group)
    parts = out.view(world, y2.shape[0], cq + 2 * ck).split([cq, ck, ck], dim=-1)
    return tuple(p.permute(1, 0, 2).reshape(*lead, world * p.shape[-1]) for p in parts)


def _fused_peer(site, x: torch.Tensor, n_out: int, parts, int8: bool, call):
    """Run the projection with its all-gather fused in (the ``b200mm_*_peer``
    entry points: the kernel stores into every rank's gathered buffer) when
    the call is in the fused regime -- up to 32 token rows for int8 weights,
    8 for 16-bit, at most the site's rows; returns the gathered tensor, or
    None for the caller's unfused path."""
    if site is None or site.ctx.world == 1 or not site.ctx.fused:
        return None
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    if (rows < 1 or rows > (32 if int8 else 8) or rows > site.max_rows or not x.is_cuda or x.dtype != site.dtype
            or n_out * site.ctx.world != site.width):
        return None
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or (x2.stride(0) * x2.element_size()) % 16 or x2.data_ptr() % 16:
        return None
    po = site.peer_out(tuple(parts))
    with _capi.on_device(x2):
        st = call(x2, rows, po)
    if st == 1:  # B200MM_ERR_SHAPE: outside the fused regime, nothing launched
        return None
    _capi.check(st, "b200mm_*_peer")
    return site.result(tuple(x.shape[:-1]), rows)


class ShardedLinear(nn.Module):
    """Bias-free projection holding this rank's block of output rows of the
    full weight; the output is gathered back to the full width."""

    def __init__(self, weight: torch.Tensor, world: int, group=None) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.world, self.group, self.site = world, group, None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if w.dtype == x.dtype and w.stride(-1) == 1:
            y = _fused_peer(self.site, x, w.shape[0], (w.shape[0],), False,
                            lambda x2, rows, po: _capi.lib.b200mm_linear_peer(
                                x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0), rows, w.shape[0], w.shape[1],
                                _capi.dtype_code(x.dtype), po, _capi.stream_of(x2)))
            if y is not None:
                return y
        return gather_cols(b200_linear(x, w), self.world, self.group, self.site)


class ShardedInt8Attention(Int8Attention):
    """``Int8Attention`` whose QKV and ``o`` projections run on this rank's
    rows; the attention core in between is the inherited, replicated one."""

    @classmethod
    def from_module(cls, att: Int8Attention, rank: int, world: int, group=None) -> "ShardedInt8Attention":
        if att.num_heads % world or att.num_kv_heads % world:
            raise ValueError(f"{att.num_heads} q / {att.num_kv_heads} kv heads do not split over {world} ranks")
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        for name in ("hidden_size", "num_heads", "num_kv_heads", "head_dim", "n_q", "n_k"):
            setattr(out, name, getattr(att, name))
        rows = torch.tensor(qkv_rows(att.n_q, att.n_k, rank, world), device=att.q_qkv.device)
        out.register_buffer("q_qkv", att.q_qkv.index_select(0, rows).contiguous())
        out.register_buffer("s_qkv", att.s_qkv.index_select(0, rows).contiguous())
        hid = even_range(att.o.weight.shape[0], rank, world)
        out.o = ShardedLinear(att.o.weight.detach()[hid.start:hid.stop].contiguous(), world, group)
        out.q_norm, out.k_norm = att.q_norm, att.k_norm
        out.decode_attn_op = getattr(att, "decode_attn_op", None)
        out.world, out.group, out.site = world, group, None
        return out

    def project_qkv(self, x: torch.Tensor):
        cq, ck, q, s = self.n_q // self.world, self.n_k // self.world, self.q_qkv, self.s_qkv
        y = _fused_peer(self.site, x, q.shape[0], (cq, ck, ck), True,
                        lambda x2, rows, po: _capi.lib.b200mm_linear_w8_peer(
                            x2.data_ptr(), x2.stride(0), q.data_ptr(), s.data_ptr(), q.stride(0), rows, q.shape[0],
                            q.shape[1], _capi.dtype_code(x.dtype), po, _capi.stream_of(x2)))
        if y is not None:
            return y.split([self.world * cq, self.world * ck, self.world * ck], dim=-1)
        y = int8_linear(x, q, s)
        return gather_qkv(y, cq, ck, self.world, self.group, self.site)


class ShardedInt8FFN(Int8FFN):
    """``Int8FFN`` with this rank's intermediate columns of gate / up and its
    hidden columns of ``down``."""

    @classmethod
    def from_module(cls, ffn: Int8FFN, rank: int, world: int, group=None) -> "ShardedInt8FFN":
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        cols = even_range(ffn.qg.shape[0], rank, world)
        sl = slice(cols.start, cols.stop)
        for name in ("qg", "sg", "qu", "su"):
            out.register_buffer(name, getattr(ffn, name)[sl].contiguous())
        w = ffn.down.weight.detach()
        hid = even_range(w.shape[0], rank, world)
        out.down = ShardedLinear(w[hid.start:hid.stop].contiguous(), world, group)
        out.world, out.group, out.site = world, group, None
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        qg, sg, qu, su = self.qg, self.sg, self.qu, self.su
        h = _fused_peer(self.site, x, qg.shape[0], (qg.shape[0],), True,
                        lambda x2, rows, po: _capi.lib.b200mm_gate_up_silu_w8_peer(
                            x2.data_ptr(), x2.stride(0), qg.data_ptr(), sg.data_ptr(), qu.data_ptr(), su.data_ptr(),
                            qg.stride(0), rows, qg.shape[0], qg.shape[1], _capi.dtype_code(x.dtype), po,
                            _capi.stream_of(x2)))
        if h is None:
            h = gather_cols(int8_fused_gate_up_silu(x, qg, sg, qu, su), self.world, self.group, self.site)
        return self.down(h)


def peer_bytes(model: nn.Module, max_rows: int) -> int:
    """Bytes of gathered output one decode step of ``model`` needs at up to
    ``max_rows`` tokens (four call sites per layer, 256-byte aligned)."""
    total = 0
    for block in model.layers:
        att, ffn = block.attn, block.ffn
        inter = ffn.qg.shape[0] if hasattr(ffn, "qg") else ffn.gate.weight.shape[0]
        esz = 2
        for width in (att.n_q + 2 * att.n_k, att.hidden_size, inter, att.hidden_size):
            total += (max_rows * width * esz + 255) // 256 * 256
    vocab = model.lm_head.weight.shape[0]
    return total + (max_rows * vocab * 2 + 255) // 256 * 256


def shard_decode_model(model: nn.Module, rank: int, world: int, group=None, peer=None,
                       max_rows: int = 64, lm_head: bool = True) -> nn.Module:
    """Replace every layer's int8 attention / FFN with its column-sharded
    form (in place; the full projection weights are dropped), and with
    ``lm_head`` the LM head by vocabulary rows (the logits gathered).  With
    ``peer`` (a ``peer.PeerGather`` of at least ``peer_bytes(model,
    max_rows)``), the gathers of up to ``max_rows`` tokens run over peer
    memory, one call-site region each.  Returns ``model``."""
    dtype = model.layers[0].attn.o.weight.dtype
    for block in model.layers:
        att = ShardedInt8Attention.from_module(block.attn, rank, world, group)
        ffn = ShardedInt8FFN.from_module(block.ffn, rank, world, group)
        if peer is not None:
            inter = ffn.qg.shape[0] * world
            att.site = peer.site(max_rows, att.n_q + 2 * att.n_k, dtype)
            att.o.site = peer.site(max_rows, att.hidden_size, dtype)
            ffn.site = peer.site(max_rows, inter, dtype)
            ffn.down.site = peer.site(max_rows, att.hidden_size, dtype)
        block.attn, block.ffn = att, ffn
    if lm_head:
        w = model.lm_head.weight.detach()
        rows = even_range(w.shape[0], rank, world)
        head = ShardedLinear(w[rows.start:rows.stop].contiguous(), world, group)
        if peer is not None:
            head.site = peer.site(max_rows, w.shape[0], w.dtype)
        model.lm_head = head
    return model


__all__ = ["ShardedInt8Attention", "ShardedInt8FFN", "ShardedLinear", "even_range", "gather_cols",
           "gather_qkv", "peer_bytes", "qkv_rows", "shard_decode_model"]
