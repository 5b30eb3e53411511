"""Absorbed latent-KV MLA decode backend for the engine's ``MLAttention``.

The reference decode step (engine/mla.py:173-265, T == 1) re-expands K and V
for every cached token on every step.  This backend keeps the reference's
cache (``MLAKVCache``: ``c_kv`` and ``k_rope_pre``, engine/mla.py:41-87) and
its module parameters, and runs the attention core in one pass over the
latent cache through ``b200mm_mla_decode``:

* two per-token side-bands are attached to the cache object and filled once
  per token by ``b200mm_mla_append`` (lazily for tokens a prefill wrote, and
  for the new token of each decode step): the k-RMS factor ``kscale[B, S, KV]``
  (fp32; the scalar the ``k_norm`` RMSNorm multiplies each reconstructed K
  head by) and the RoPE'd, k_norm-weighted rope half of K, ``kz[B, S, KV, DR]``
  (model dtype).  A decode step therefore reads the latent, ``kz`` and
  ``kscale`` -- the same 1056 bytes per token as latent + ``k_rope_pre`` +
  ``kscale`` -- and never rotates keys;
* the query is absorbed through ``W_uk`` and the context is split across CTAs
  with an online-softmax merge; ``W_uv`` is applied once per head.

Public pieces:
  mla_decode(...)       functional core (q already q_norm'ed)
  mla_append(...)       side-band fill for a token range
  mla_sidebands(...)    allocate + fill both side-bands for positions [0, L)
  B200MLAttention       drop-in module (same constructor / forward signature
                        as the reference ``MLAttention``)
  apply_b200_mla(model) in-place swap walker, mirroring ``apply_mla``
                        (mla/swap.py:21-69)
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F
from torch import nn

from . import _capi
from .kernels._eager import RMSNorm, rotate_half
from .kernels.linear import b200_linear


def rope_inv_freq(head_dim: int, d_rope: int, theta: float, device=None) -> torch.Tensor:
    """The reference's partial-RoPE frequencies (engine/mla.py:158-163): the
    first d_rope/2 entries of the head_dim-sized vector, in float32."""
    full = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    return full[: d_rope // 2].contiguous().to(device)


def _shape(B, H, KV, D, DR, R, dtype, eps) -> _capi.MlaShape:
    return _capi.MlaShape(B=B, H=H, KV=KV, D=D, DR=DR, R=R, dtype=_capi.dtype_code(dtype), eps=eps)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def batch_shard(B: int, world: int, rank: int) -> range:
    """Batch rows of an MLA decode that GPU `rank` of `world` serves.

    MLA decode shards by batch row with no collective: each GPU streams only
    its own rows' latent cache (the rows are independent), and outputs are
    gathered afterwards if the caller needs them on one GPU.  Rank r takes
    rows [B*r/world, B*(r+1)/world); with B < world the surplus ranks get an
    empty range and idle (their GB/s counts as zero in an aggregate)."""
    if world < 1 or not 0 <= rank < world or B < 0:
        raise ValueError(f"bad shard request: B={B} world={world} rank={rank}")
    return range(B * rank // world, B * (rank + 1) // world)


def decode_shard(B: int, L: int, world: int, rank: int) -> tuple[range, range]:
    """Batch rows and context tokens of an MLA decode step that GPU ``rank`` of
    ``world`` serves.  With ``B >= world``: a batch-row split (``batch_shard``),
    each rank its rows' whole context, no collective.  With fewer rows than
    GPUs: a context split -- every rank streams its slice
    ``[L*r/world, L*(r+1)/world)`` of every row's cache
    (``mla_decode_partial``), and the slices' partial softmaxes meet in one
    small exchange (one all-gather of B x H x (R + 2) floats per rank) before
    the W_uv step (``mla_combine_partials``): the flash-decoding split, across
    GPUs."""
    if world < 1 or not 0 <= rank < world or B < 0 or L < 1:
        raise ValueError(f"bad shard request: B={B} L={L} world={world} rank={rank}")
    if B >= world or B == 0:
        return batch_shard(B, world, rank), range(0, L)
    if L < world:
        raise ValueError(f"a context of {L} tokens cannot be split over {world} GPUs")
    return range(0, B), range(L * rank // world, L * (rank + 1) // world)


def partial_numel(B: int, H: int, R: int) -> int:
    """fp32 elements of one partial decode: av [B, H, R] then ml [B, H, 2]."""
    return B * H * (R + 2)


def mla_decode_partial(q: torch.Tensor, c_kv: torch.Tensor, kz: torch.Tensor | None, kscale: torch.Tensor,
                       w_uk: torch.Tensor | None, k_norm_w: torch.Tensor, inv_freq: torch.Tensor | None, *,
                       num_kv_heads: int, L: int, tokens: range, scale: float, eps: float,
                       out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The decode step over cache tokens ``tokens`` only, for a query at
    position ``L - 1``: returns one flat fp32 buffer of ``partial_numel``
    elements -- ``av`` (B, H, R), the latent mixed by the softmax over those
    tokens, then ``ml`` (B, H, 2), their max score and sum of exp -- so one
    all-gather moves a rank's whole partial.  No W_uv step:
    ``mla_combine_partials`` merges the ranges."""
    B, H, D = q.shape
    R = c_kv.shape[-1]
    DR = 0 if kz is None else kz.shape[-1]
    _capi.require_cuda(q, c_kv, kscale)
    if q.stride(-1) != 1 or q.stride(1) != D:
        q = q.contiguous()
    shp = _shape(B, H, num_kv_heads, D, DR, R, q.dtype, eps)
    n = len(tokens)
    ws_bytes = int(_capi.lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), max(n, 1)))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    numel = partial_numel(B, H, R)
    if out is None:
        out = torch.empty(numel, dtype=torch.float32, device=q.device)
    if out.dtype != torch.float32 or out.numel() != numel or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous float32 buffer of {numel} elements")
    with _capi.on_device(q):
        st = _capi.lib.b200mm_mla_decode_partial(
            ctypes.byref(shp), q.data_ptr(), q.stride(0), c_kv.data_ptr(), c_kv.stride(0), c_kv.stride(1),
            _ptr(kz), 0 if kz is None else kz.stride(0), 0 if kz is None else kz.stride(1),
            kscale.data_ptr(), kscale.stride(0), kscale.stride(1), _ptr(w_uk), k_norm_w.data_ptr(), _ptr(inv_freq),
            float(scale), L, tokens.start, tokens.stop, out.data_ptr(), out.data_ptr() + 4 * B * H * R,
            workspace.data_ptr(), workspace.numel(), _capi.stream_of(q))
    _capi.check(st, "b200mm_mla_decode_partial")
    return out


def mla_combine_partials(parts: torch.Tensor, w_uv: torch.Tensor, *, batch: int, num_heads: int, head_dim: int,
                         d_rope: int, dtype: torch.dtype, eps: float, out: torch.Tensor | None = None,
                         workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Merge the partial decodes of ``n`` token ranges -- ``parts`` (n,
    partial_numel) fp32, one row per range as ``mla_decode_partial`` wrote
    them (an all-gather of the ranks' buffers) -- and apply W_uv: the decode
    output (batch, num_heads, head_dim) in ``dtype``."""
    n = parts.shape[0]
    KV, _, R = w_uv.shape
    B, H = batch, num_heads
    _capi.require_cuda(parts, w_uv)
    if parts.dtype != torch.float32 or parts.dim() != 2 or parts.shape[1] != partial_numel(B, H, R) \
            or parts.stride(1) != 1:
        raise ValueError(f"parts must be float32 (n, {partial_numel(B, H, R)}) with unit inner stride")
    shp = _shape(B, H, KV, head_dim, d_rope, R, dtype, eps)
    ws_bytes = int(_capi.lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), 1))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=parts.device)
    if out is None:
        out = torch.empty((B, H, head_dim), dtype=dtype, device=parts.device)
    with _capi.on_device(parts):
        st = _capi.lib.b200mm_mla_combine_partials(
            ctypes.byref(shp), parts.data_ptr(), parts.stride(0), parts.data_ptr() + 4 * B * H * R, parts.stride(0),
            n, w_uv.data_ptr(), out.data_ptr(), out.stride(0), workspace.data_ptr(), workspace.numel(),
            _capi.stream_of(parts))
    _capi.check(st, "b200mm_mla_combine_partials")
    return out


def workspace_bytes(B: int, H: int, KV: int, D: int, DR: int, R: int, L: int, dtype, eps: float = 1e-6) -> int:
    shp = _shape(B, H, KV, D, DR, R, dtype, eps)
    return int(_capi.lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L))


def mla_append(c_kv: torch.Tensor, k_rope_pre: torch.Tensor | None, w_uk: torch.Tensor | None,
               k_norm_w: torch.Tensor, inv_freq: torch.Tensor | None, kscale: torch.Tensor,
               kz: torch.Tensor | None, *, B: int, t0: int, t1: int, num_kv_heads: int, head_dim: int,
               eps: float) -> None:
    """Fill the side-bands ``kscale[:B, t0:t1]`` and ``kz[:B, t0:t1]``.

    c_kv [*, S, R]; k_rope_pre, kz [*, S, KV, DR] or None (DR == 0);
    w_uk [KV, DN, R] or None (DN == 0); k_norm_w fp32 [D]; inv_freq fp32
    [DR/2]; kscale fp32 [*, S, KV].
    """
    _capi.require_cuda(c_kv, kscale)
    R = c_kv.shape[-1]
    DR = 0 if k_rope_pre is None else k_rope_pre.shape[-1]
    shp = _shape(B, num_kv_heads, num_kv_heads, head_dim, DR, R, c_kv.dtype, eps)
    if kscale.dtype != torch.float32 or kscale.stride(-1) != 1:
        raise ValueError("kscale must be float32 with a dense last dim")
    with _capi.on_device(c_kv):
        st = _capi.lib.b200mm_mla_append(
            ctypes.byref(shp), c_kv.data_ptr(), c_kv.stride(0), c_kv.stride(1),
            _ptr(k_rope_pre), 0 if k_rope_pre is None else k_rope_pre.stride(0),
            0 if k_rope_pre is None else k_rope_pre.stride(1),
            _ptr(w_uk), k_norm_w.data_ptr(), _ptr(inv_freq),
            kscale.data_ptr(), kscale.stride(0), kscale.stride(1),
            _ptr(kz), 0 if kz is None else kz.stride(0), 0 if kz is None else kz.stride(1),
            t0, t1, _capi.stream_of(c_kv),
        )
    _capi.check(st, "b200mm_mla_append")


def mla_sidebands(c_kv: torch.Tensor, k_rope_pre: torch.Tensor | None, w_uk: torch.Tensor | None,
                  k_norm_w: torch.Tensor, inv_freq: torch.Tensor | None, *, B: int, L: int, num_kv_heads: int,
                  head_dim: int, eps: float):
    """Allocate the two side-bands for a cache of ``c_kv.shape[1]`` positions
    and fill positions ``[0, L)`` of rows ``0..B-1``.  Returns (kscale, kz)."""
    S = c_kv.shape[1]
    DR = 0 if k_rope_pre is None else k_rope_pre.shape[-1]
    kscale = torch.empty((c_kv.shape[0], S, num_kv_heads), dtype=torch.float32, device=c_kv.device)
    kz = torch.empty((c_kv.shape[0], S, num_kv_heads, DR), dtype=c_kv.dtype, device=c_kv.device) if DR else None
    mla_append(c_kv, k_rope_pre, w_uk, k_norm_w, inv_freq, kscale, kz, B=B, t0=0, t1=L,
               num_kv_heads=num_kv_heads, head_dim=head_dim, eps=eps)
    return kscale, kz


def mla_decode(q: torch.Tensor, c_kv: torch.Tensor, kz: torch.Tensor | None, kscale: torch.Tensor,
               w_uk: torch.Tensor | None, w_uv: torch.Tensor, k_norm_w: torch.Tensor,
               inv_freq: torch.Tensor | None, *, L: int, scale: float, eps: float,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One MLA decode step over cache positions ``0..L-1``.

    Args:
        q: ``(B, H, D)`` query after ``q_norm``, before RoPE.
        c_kv: ``(*, S, R)`` latent cache (rows ``0..B-1`` used), S >= L.
        kz: ``(*, S, KV, DR)`` RoPE'd key side-band, or None if DR == 0.
        kscale: ``(*, S, KV)`` float32 side-band; both valid for positions < L.
        w_uk: ``(KV, DN, R)``, or None if DN == 0.  w_uv: ``(KV, D, R)``.
        k_norm_w: ``(D,)`` float32.  inv_freq: ``(DR/2,)`` float32.
    Returns:
        ``(B, H, D)`` attention output in q's dtype (the input of ``o``).
    """
    B, H, D = q.shape
    R = c_kv.shape[-1]
    KV = w_uv.shape[0]
    DR = 0 if kz is None else kz.shape[-1]
    _capi.require_cuda(q, c_kv, kscale, w_uv)
    if q.stride(-1) != 1 or q.stride(1) != D:
        q = q.contiguous()
    shp = _shape(B, H, KV, D, DR, R, q.dtype, eps)
    ws_bytes = int(_capi.lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=q.device)
    with _capi.on_device(q):
        st = _capi.lib.b200mm_mla_decode(
            ctypes.byref(shp), q.data_ptr(), q.stride(0),
            c_kv.data_ptr(), c_kv.stride(0), c_kv.stride(1),
            _ptr(kz), 0 if kz is None else kz.stride(0), 0 if kz is None else kz.stride(1),
            kscale.data_ptr(), kscale.stride(0), kscale.stride(1),
            _ptr(w_uk), w_uv.data_ptr(), k_norm_w.data_ptr(), _ptr(inv_freq),
            float(scale), L, out.data_ptr(), out.stride(0),
            workspace.data_ptr(), workspace.numel(), _capi.stream_of(q),
        )
    _capi.check(st, "b200mm_mla_decode")
    return out


# ---------------------------------------------------------------------------
# drop-in module
# ---------------------------------------------------------------------------
def _sideband(kv_cache, layer_idx: int, KV: int, DR: int):
    """The side-bands of ``layer_idx`` (allocated on first use): fp32 ``kscale``
    [max_batch, S, KV], ``kz`` [max_batch, S, KV, DR] in the cache dtype (None
    if DR == 0), and the dict of how many leading positions they cover."""
    bands = getattr(kv_cache, "_b200_kscale", None)
    if bands is None:
        bands = {}
        kv_cache._b200_kscale = bands
        kv_cache._b200_kz = {}
        kv_cache._b200_kscale_len = {}
    if layer_idx not in bands:
        c = kv_cache.c_kv[layer_idx]
        bands[layer_idx] = torch.empty((c.shape[0], c.shape[1], KV), dtype=torch.float32, device=c.device)
        kv_cache._b200_kz[layer_idx] = (
            torch.empty((c.shape[0], c.shape[1], KV, DR), dtype=c.dtype, device=c.device) if DR > 0 else None)
        kv_cache._b200_kscale_len[layer_idx] = 0
    return bands[layer_idx], kv_cache._b200_kz[layer_idx], kv_cache._b200_kscale_len


class B200MLAttention(nn.Module):
    """Partial-RoPE GQA over the compressed latent cache, with the T == 1
    (decode) step on the absorbed B200 kernel.

    Constructor, parameters (``q, dkv, uk_nope, uv, kr, o, q_norm, k_norm``,
    ``rope_cos/rope_sin`` buffers) and ``forward`` signature follow the
    reference ``MLAttention`` (engine/mla.py:105-181).  Prefill (T > 1)
    follows the reference's reconstruct-then-SDPA math (engine/mla.py:189-265).
    """

    def __init__(self, *, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int, rms_eps: float,
                 rank: int, d_rope: int, max_position_embeddings: int, rope_theta: float = 10000.0,
                 qk_norm_mode: str = "single") -> None:
        super().__init__()
        if d_rope < 0 or d_rope > head_dim:
            raise ValueError(f"d_rope={d_rope} not in [0, head_dim={head_dim}]")
        if qk_norm_mode != "single":
            raise NotImplementedError(f"qk_norm_mode={qk_norm_mode!r}: only 'single' is implemented")
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.rank, self.d_rope, self.d_nope = rank, d_rope, head_dim - d_rope
        self.qk_norm_mode = qk_norm_mode
        self.rope_theta = rope_theta
        self.q = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.dkv = nn.Linear(hidden_size, rank, bias=False)
        self.uk_nope = nn.Linear(rank, num_kv_heads * self.d_nope, bias=False) if self.d_nope > 0 else None
        self.uv = nn.Linear(rank, num_kv_heads * head_dim, bias=False)
        self.kr = nn.Linear(hidden_size, num_kv_heads * d_rope, bias=False) if d_rope > 0 else None
        self.o = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        self.q_norm = RMSNorm(head_dim, rms_eps)
        self.k_norm = RMSNorm(head_dim, rms_eps)
        if d_rope > 0:
            inv = rope_inv_freq(head_dim, d_rope, rope_theta)
            ang = torch.outer(torch.arange(max_position_embeddings, dtype=torch.float32), inv)
            emb = torch.cat([ang, ang], dim=-1)
            self.register_buffer("rope_cos", emb.cos(), persistent=False)
            self.register_buffer("rope_sin", emb.sin(), persistent=False)
        else:
            self.rope_cos = None
            self.rope_sin = None

    @classmethod
    def from_eager(cls, eager: nn.Module, *, rope_theta: float | None = None) -> "B200MLAttention":
        """Wrap a reference ``MLAttention``, sharing all parameters and buffers.

        The reference module does not store its RoPE base; pass ``rope_theta``
        (the artifact's ``meta["rope_theta"]``) unless ``eager`` carries one.
        """
        theta = rope_theta if rope_theta is not None else getattr(eager, "rope_theta", None)
        if eager.d_rope > 0 and theta is None:
            raise ValueError("rope_theta is required to wrap an MLAttention with d_rope > 0")
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        for name in ("num_heads", "num_kv_heads", "head_dim", "rank", "d_rope", "d_nope", "qk_norm_mode"):
            setattr(out, name, getattr(eager, name))
        out.rope_theta = theta
        for name in ("q", "dkv", "uk_nope", "uv", "kr", "o", "q_norm", "k_norm"):
            setattr(out, name, getattr(eager, name))
        out.rope_cos = eager.rope_cos
        out.rope_sin = eager.rope_sin
        # the wrapped module serves the prefill; kept outside the module tree
        # (its parameters are already registered here under the same names)
        out.__dict__["_b200_reference"] = eager
        return out

    # -- helpers ------------------------------------------------------------
    def _consts(self, device):
        """float32 k_norm weight and RoPE frequencies, cached per device."""
        key = (device, self.k_norm.weight._version, self.k_norm.weight.data_ptr())
        cache = getattr(self, "_b200_consts", None)
        if cache is None or cache[0] != key:
            kw = self.k_norm.weight.detach().float().contiguous().to(device)
            inv = rope_inv_freq(self.head_dim, self.d_rope, self.rope_theta, device) if self.d_rope > 0 else None
            cache = (key, kw, inv)
            self._b200_consts = cache
        return cache[1], cache[2]

    def _q_latent_weight(self, x: torch.Tensor) -> torch.Tensor | None:
        """``[q; dkv; kr]`` row-stacked in one buffer (the fused "Q + latent"
        projection of the decode step, replacing the three Linears at
        engine/mla.py:195-205).  Built once: the three weights are rebound as
        views of the buffer, so no weight is stored twice and state dicts
        keep their keys.  Rebuilt if a weight was replaced since (``.to()``,
        a new Parameter); None when the weights cannot serve ``x``."""
        lins = [self.q, self.dkv] + ([self.kr] if self.kr is not None else [])
        if any(lin.bias is not None or lin.weight.dtype != x.dtype or lin.weight.device != x.device
               for lin in lins):
            return None
        W = getattr(self, "_b200_qlat", None)
        if W is not None and W.dtype == x.dtype and W.device == x.device:
            off, ok = 0, True
            for lin in lins:
                w = lin.weight
                ok = ok and w.data_ptr() == W[off:].data_ptr() and w.shape[0] + off <= W.shape[0] and w.is_contiguous()
                off += w.shape[0]
            if ok and off == W.shape[0]:
                return W
        with torch.no_grad():
            W = torch.cat([lin.weight.detach() for lin in lins], 0).contiguous()
            off = 0
            for lin in lins:
                n = lin.weight.shape[0]
                lin.weight = nn.Parameter(W[off:off + n], requires_grad=lin.weight.requires_grad)
                off += n
        self._b200_qlat = W
        return W

    def supports_fast_decode(self, x: torch.Tensor) -> bool:
        return x.is_cuda and x.shape[1] == 1 and x.dtype in _capi.DTYPE_CODES

    def forward(self, x: torch.Tensor, *, kv_cache, layer_idx: int, start_pos: int,
                cos: torch.Tensor | None = None, sin: torch.Tensor | None = None) -> torch.Tensor:
        """T == 1 (decode): the absorbed B200 kernels.  T > 1 (prefill): the
        reference's reconstruct-then-SDPA math, on purpose -- the north-star
        path is the decode step; a prefill writes the cache once and its
        side-bands are filled lazily by the next decode.  When this module
        wraps a reference ``MLAttention`` (``from_eager``), the prefill is
        that module's own ``forward``.  There is no CPU path: CPU tensors and
        dtypes the kernels do not take raise."""
        del cos, sin  # accepted for signature compatibility, as in the reference
        _capi.require_cuda(x)
        if x.dtype not in _capi.DTYPE_CODES:
            raise ValueError(f"B200MLAttention takes float32 / float16 / bfloat16 inputs, got {x.dtype}")
        if x.shape[1] == 1:
            return self._decode(x, kv_cache=kv_cache, layer_idx=layer_idx, start_pos=start_pos)
        return self._prefill(x, kv_cache=kv_cache, layer_idx=layer_idx, start_pos=start_pos)

    def _prefill(self, x, *, kv_cache, layer_idx, start_pos):
        # tokens rewritten here invalidate their side-band entries
        lens = getattr(kv_cache, "_b200_kscale_len", None)
        if lens is not None and layer_idx in lens:
            lens[layer_idx] = min(lens[layer_idx], start_pos)
        ref = self.__dict__.get("_b200_reference")
        if ref is not None:
            return ref(x, kv_cache=kv_cache, layer_idx=layer_idx, start_pos=start_pos)
        return self._eager(x, kv_cache=kv_cache, layer_idx=layer_idx, start_pos=start_pos)

    def _write_cache(self, x, kv_cache, layer_idx, start_pos, end):
        B, T, _ = x.shape
        kv_cache.c_kv[layer_idx][:B, start_pos:end, :] = self.dkv(x)
        if self.d_rope > 0:
            kv_cache.k_rope_pre[layer_idx][:B, start_pos:end] = self.kr(x).view(B, T, self.num_kv_heads, self.d_rope)

    def _decode(self, x, *, kv_cache, layer_idx, start_pos):
        B = x.shape[0]
        H, KV, D, DR, DN = self.num_heads, self.num_kv_heads, self.head_dim, self.d_rope, self.d_nope
        end = start_pos + 1
        W = self._q_latent_weight(x)
        if W is not None:  # one launch for q, the latent c_kv and the pre-RoPE key
            y = b200_linear(x, W)
            q, c_new, k_new = y.split([H * D, self.rank, KV * DR], dim=-1)
            kv_cache.c_kv[layer_idx][:B, start_pos:end, :] = c_new
            if DR > 0:
                kv_cache.k_rope_pre[layer_idx][:B, start_pos:end] = k_new.view(B, 1, KV, DR)
            q = self.q_norm(q.reshape(B, 1, H, D))
        else:
            q = self.q_norm(self.q(x).view(B, 1, H, D))
            self._write_cache(x, kv_cache, layer_idx, start_pos, end)
        c = kv_cache.c_kv[layer_idx]
        kr = kv_cache.k_rope_pre[layer_idx] if DR > 0 else None
        w_uk = self.uk_nope.weight.view(KV, DN, self.rank) if DN > 0 else None
        w_uv = self.uv.weight.view(KV, D, self.rank)
        kscale, kz, lens = _sideband(kv_cache, layer_idx, KV, DR)
        valid = min(lens[layer_idx], start_pos)
        kw, inv = self._consts(x.device)
        mla_append(c, kr, w_uk, kw, inv, kscale, kz, B=B, t0=valid, t1=end, num_kv_heads=KV, head_dim=D,
                   eps=self.k_norm.eps)
        lens[layer_idx] = end
        attn = mla_decode(q.view(B, H, D), c, kz, kscale, w_uk, w_uv, kw, inv, L=end, scale=D ** -0.5,
                          eps=self.k_norm.eps)
        return self.o(attn.view(B, 1, H * D))

    def _eager(self, x, *, kv_cache, layer_idx, start_pos):
        """Reconstruct-then-SDPA path of the reference (engine/mla.py:189-265)."""
        B, T, _ = x.shape
        H, KV, D, DN, DR = self.num_heads, self.num_kv_heads, self.head_dim, self.d_nope, self.d_rope
        end = start_pos + T
        q = self.q_norm(self.q(x).view(B, T, H, D)).transpose(1, 2)
        self._write_cache(x, kv_cache, layer_idx, start_pos, end)
        c = kv_cache.c_kv[layer_idx][:B, :end]
        v = self.uv(c).view(B, end, KV, D)
        parts = []
        if DN > 0:
            parts.append(self.uk_nope(c).view(B, end, KV, DN))
        if DR > 0:
            parts.append(kv_cache.k_rope_pre[layer_idx][:B, :end])
        k = self.k_norm(torch.cat(parts, dim=-1) if len(parts) > 1 else parts[0])
        if DR > 0:
            qn, qr = q.split([DN, DR], dim=-1)
            kn, kr = k.split([DN, DR], dim=-1)
            cq, sq = self.rope_cos[start_pos:end].to(q.dtype), self.rope_sin[start_pos:end].to(q.dtype)
            ck, sk = self.rope_cos[:end].to(k.dtype), self.rope_sin[:end].to(k.dtype)
            qr = qr * cq + rotate_half(qr) * sq
            kr = kr.transpose(1, 2)
            kr = (kr * ck + rotate_half(kr) * sk).transpose(1, 2)
            q = torch.cat([qn, qr], dim=-1) if DN > 0 else qr
            k = torch.cat([kn, kr], dim=-1) if DN > 0 else kr
        k = k.transpose(1, 2)
        v = v.transpose(1, 2)
        if H // KV > 1:
            k = k.repeat_interleave(H // KV, dim=1)
            v = v.repeat_interleave(H // KV, dim=1)
        qp = torch.arange(start_pos, end, device=x.device).unsqueeze(1)
        kp = torch.arange(0, end, device=x.device).unsqueeze(0)
        attn = F.scaled_dot_product_attention(q, k, v, attn_mask=qp >= kp)
        return self.o(attn.transpose(1, 2).reshape(B, T, H * D))


def apply_b200_mla(model: nn.Module, *, rope_theta: float | None = None) -> nn.Module:
    """Swap every latent-attention ``block.attn`` (anything with ``dkv``,
    ``uv`` and ``rank``) for :class:`B200MLAttention`, sharing parameters.
    Idempotent; returns ``model``."""
    if rope_theta is None:
        cfg = getattr(model, "cfg", None)
        rp = getattr(cfg, "rope_parameters", None)
        if isinstance(rp, dict) and "rope_theta" in rp:
            rope_theta = float(rp["rope_theta"])
        elif cfg is not None and hasattr(cfg, "rope_theta"):
            rope_theta = float(cfg.rope_theta)
    for block in model.layers:
        a = block.attn
        if isinstance(a, B200MLAttention):
            continue
        if all(hasattr(a, n) for n in ("dkv", "uv", "rank")):
            block.attn = B200MLAttention.from_eager(a, rope_theta=rope_theta)
    return model
