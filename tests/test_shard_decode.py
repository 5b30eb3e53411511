"""Host logic of the column-sharded decode step (``llms_b200.shard``): the
row blocks each rank takes, and the all-gather + reorder that rebuilds the
unsharded activations -- on CPU with two and four gloo ranks, with plain
matmuls standing in for the kernels."""

import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from llms_b200.shard import even_range, qkv_rows


def test_even_range_and_qkv_rows_partition():
    for world in (1, 2, 4, 8):
        cols = [c for r in range(world) for c in even_range(12288, r, world)]
        assert cols == list(range(12288))
        rows = [q for r in range(world) for q in qkv_rows(4096, 1024, r, world)]
        assert sorted(rows) == list(range(6144))
        # rank r's q rows are whole heads: [r*4096/world, (r+1)*4096/world)
        r0 = qkv_rows(4096, 1024, 1 % world, world)
        assert r0[0] == (1 % world) * 4096 // world and (r0[0] % 128) == 0
    with pytest.raises(ValueError):
        even_range(100, 0, 3)
    with pytest.raises(ValueError):
        even_range(12, 2, 2)


def _worker(rank, world, port, out):
    import torch.distributed as dist
    from llms_b200.shard import gather_cols, gather_qkv
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        nq, nk, C, I = 64, 16, 32, 96
        x = torch.randn(3, 2, C, generator=g)
        w_qkv = torch.randn(nq + 2 * nk, C, generator=g)
        w_gu = torch.randn(2, I, C, generator=g)
        w_o = torch.randn(C, nq, generator=g)
        # QKV: local head-aligned rows, gathered and reordered
        rows = torch.tensor(qkv_rows(nq, nk, rank, world))
        q, k, v = gather_qkv(x @ w_qkv[rows].T, nq // world, nk // world, world)
        full = x @ w_qkv.T
        ok = [torch.allclose(q, full[..., :nq]), torch.allclose(k, full[..., nq:nq + nk]),
              torch.allclose(v, full[..., nq + nk:])]
        # gate-up by intermediate columns, then the gathered intermediate
        cols = even_range(I, rank, world)
        sl = slice(cols.start, cols.stop)
        h = torch.nn.functional.silu(x @ w_gu[0, sl].T) * (x @ w_gu[1, sl].T)
        hf = torch.nn.functional.silu(x @ w_gu[0].T) * (x @ w_gu[1].T)
        ok.append(torch.allclose(gather_cols(h, world), hf))
        # o by hidden columns
        hid = even_range(C, rank, world)
        y = gather_cols(full[..., :nq] @ w_o[hid.start:hid.stop].T, world)
        ok.append(torch.allclose(y, full[..., :nq] @ w_o.T, atol=1e-4))
        out.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_projections_gather_to_full_gloo(world):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29600 + world + (os.getpid() % 200)
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert sorted(res) == list(range(world))
    for r, ok in res.items():
        assert all(ok), (r, ok)


def test_peer_sites_fit_peer_bytes():
    """shard_decode_model with a peer context reserves one region per call
    site (QKV, o, gate-up, down per layer, then the LM head), each as wide as
    the gathered output, and peer_bytes covers them all (CPU: a recording
    stand-in for the symmetric buffer)."""
    import dataclasses

    from llms_b200.qwen3 import QWEN3_8B, synthetic_int8_model
    from llms_b200.shard import peer_bytes, shard_decode_model

    shape = dataclasses.replace(QWEN3_8B, hidden_size=256, num_attention_heads=4, num_key_value_heads=2,
                                head_dim=64, intermediate_size=512, vocab_size=1024, num_hidden_layers=2)
    model = synthetic_int8_model(shape, device="cpu")
    need = peer_bytes(model, 8)

    class Ctx:
        world = 2

        def __init__(self):
            self.sites = []

        def site(self, rows, width, dtype):
            self.sites.append((rows, width, dtype))
            return ("site", len(self.sites))

    ctx = Ctx()
    shard_decode_model(model, 0, 2, peer=ctx, max_rows=8)
    widths = [w for _, w, _ in ctx.sites]
    qkv = 4 * 64 + 2 * 2 * 64
    assert widths == [qkv, 256, 512, 256] * 2 + [1024]
    assert all(r == 8 and d == torch.bfloat16 for r, _, d in ctx.sites)
    assert sum((8 * w * 2 + 255) // 256 * 256 for w in widths) <= need
    assert model.lm_head.weight.shape == (512, 256)  # vocabulary rows of rank 0
