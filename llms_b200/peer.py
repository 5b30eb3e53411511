"""Peer-memory all-gather for the column-sharded decode step.

``PeerGather`` owns one buffer per rank in torch's symmetric memory (every
rank's buffer mapped into every other rank's address space over NVLink; the
mapping is torch's plumbing) and hands out per-call-site regions of it.
``PeerGather.gather`` is one ``b200mm_peer_gather`` launch: this rank's column
block goes straight into every rank's region at its final column position,
and the kernel returns once every rank's block has arrived -- the NCCL
all-gather plus the permute that followed it, in one kernel.

Each call site (``site = ctx.site(max_rows, width)``) has its own region, so
a gathered result stays valid until the same site gathers again (the next
decode step).  Rows beyond the site's ``max_rows`` are not supported: the
sharded modules fall back to the NCCL gather for them.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _capi

NCTAS = 16  # CTAs per gather launch (= flag columns); fixed for the buffer's life


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerSite:
    """One call site's region of the gathered buffer: up to ``max_rows`` rows
    of ``width`` full-width columns of ``dtype``."""

    def __init__(self, ctx: "PeerGather", offset: int, max_rows: int, width: int, dtype: torch.dtype) -> None:
        self.ctx, self.offset, self.max_rows, self.width, self.dtype = ctx, offset, max_rows, width, dtype

    def peer_out(self, parts: tuple[int, ...]) -> "_capi.PeerOut":
        """The ``b200mm_peer_out`` of this site for a shard made of ``parts``
        (cached per parts; the projection kernels write the gathered result
        here themselves)."""
        po = self._outs.get(parts) if hasattr(self, "_outs") else None
        if po is None:
            ctx = self.ctx
            po = _capi.PeerOut()
            for r in range(ctx.world):
                po.dst[r] = ctx.peer_ptrs[r] + self.offset
                po.flags[r] = ctx.fused_flag_ptrs[r]
            po.ld_dst = self.width
            for j, w in enumerate(parts):
                po.part_widths[j] = w
            po.nparts, po.rank, po.world = len(parts), ctx.rank, ctx.world
            po.ticket, po.seen, po.err = ctx.ticket_ptr, ctx.fused_seen_ptr, ctx.err_ptr
            self._outs = getattr(self, "_outs", {})
            self._outs[parts] = po
        return po

    def result(self, lead: tuple[int, ...], rows: int) -> torch.Tensor:
        """The gathered (..., width) view of this site's first ``rows`` rows."""
        esz = torch.tensor([], dtype=self.dtype).element_size()
        out = self.ctx.buf[self.offset:self.offset + rows * self.width * esz].view(self.dtype)
        return out.view(rows, self.width).view(*lead, self.width)

    def fits(self, y: torch.Tensor) -> bool:
        rows = y.numel() // y.shape[-1] if y.dim() else 0
        return (y.is_cuda and y.dtype == self.dtype and rows <= self.max_rows
                and y.shape[-1] * self.ctx.world == self.width)

    def gather(self, y: torch.Tensor, parts: tuple[int, ...] | None = None) -> torch.Tensor:
        """All-gather ``y`` (..., c) -- this rank's block, made of ``parts``
        (widths summing to c; default one part) -- into (..., world c), part j
        of every rank laid out together."""
        ctx = self.ctx
        lead, c = y.shape[:-1], y.shape[-1]
        parts = parts or (c,)
        if sum(parts) != c or not self.fits(y):
            raise ValueError(f"gather of {tuple(y.shape)} {y.dtype} does not fit the site "
                             f"({self.max_rows} rows x {self.width} {self.dtype})")
        y2 = y.reshape(-1, c)
        if y2.stride(-1) != 1:
            y2 = y2.contiguous()
        rows = y2.shape[0]
        cached = getattr(self, "_args", {}).get(parts)
        if cached is None:  # the call's pointer arrays, built once per parts
            cached = ((ctypes.c_void_p * ctx.world)(*[p + self.offset for p in ctx.peer_ptrs]),
                      (ctypes.c_int64 * len(parts))(*parts))
            self._args = getattr(self, "_args", {})
            self._args[parts] = cached
        dst, widths = cached
        with _capi.on_device(y2):
            st = _capi.lib.b200mm_peer_gather(y2.data_ptr(), y2.stride(0), rows, widths, len(parts), dst,
                                              self.width, _capi.dtype_code(y.dtype), ctx.rank, ctx.world,
                                              ctx.flag_ptrs, ctx.seen_ptr, ctx.err_ptr, NCTAS,
                                              _capi.stream_of(y2))
        _capi.check(st, "b200mm_peer_gather")
        return self.result(lead, rows)


class PeerGather:
    """The symmetric buffer of one process group: flags, then call-site
    regions.  Collective: every rank constructs it with the same arguments."""

    def __init__(self, capacity_bytes: int, group=None, device=None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group or dist.group.WORLD
        self.rank, self.world = dist.get_rank(self.group), dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError(f"b200mm_peer_gather supports up to 8 ranks, not {self.world}")
        device = torch.device(device or torch.cuda.current_device())
        # head: gather flags [world][NCTAS], seen [NCTAS], err, then the
        # fused projections' counters [8], ticket and seen
        self.flags_bytes = self.world * NCTAS * 4
        self.fused_off = self.flags_bytes + NCTAS * 4 + 4
        self.head = _align(self.fused_off + 8 * 4 + 8)
        self.capacity = _align(capacity_bytes)
        name = getattr(self.group, "group_name", None)
        if hasattr(symm_mem, "enable_symm_mem_for_group") and name is not None:
            symm_mem.enable_symm_mem_for_group(name)
        self.buf = symm_mem.empty(self.head + self.capacity, dtype=torch.uint8, device=device)
        self.buf[: self.head].zero_()
        torch.cuda.synchronize(device)
        self.handle = symm_mem.rendezvous(self.buf, name if name is not None else self.group)
        self.peer_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*self.peer_ptrs)
        base = self.buf.data_ptr()
        self.seen_ptr = base + self.flags_bytes
        self.err_ptr = base + self.flags_bytes + NCTAS * 4
        self.fused_flag_ptrs = [p + self.fused_off for p in self.peer_ptrs]
        self.ticket_ptr = base + self.fused_off + 8 * 4
        self.fused_seen_ptr = self.ticket_ptr + 4
        self._cursor = self.head
        # the sharded modules fuse a gather into its projection where they can
        # (b200mm_*_peer); False keeps projection and b200mm_peer_gather apart
        self.fused = True
        dist.barrier(group=self.group)

    def site(self, max_rows: int, width: int, dtype: torch.dtype) -> PeerSite:
        """Reserve a region for one call site: ``max_rows`` x ``width``
        (full-width) elements of ``dtype``.  Every rank must reserve the same
        sites in the same order."""
        nbytes = _align(max_rows * width * torch.tensor([], dtype=dtype).element_size())
        if self._cursor + nbytes > self.head + self.capacity:
            raise ValueError(f"peer buffer full: {self.capacity} bytes")
        s = PeerSite(self, self._cursor, max_rows, width, dtype)
        self._cursor += nbytes
        return s

    def status(self) -> int:
        """0, or 1 once a gather's wait for a peer ran out (sticky)."""
        return int(self.buf[self.flags_bytes + NCTAS * 4: self.flags_bytes + NCTAS * 4 + 4].view(torch.int32).item())


__all__ = ["NCTAS", "PeerGather", "PeerSite"]
