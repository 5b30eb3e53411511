"""MLA decode across GPUs: batch-row shards with no collective in the op
(`llms_b200.mla.batch_shard`), outputs gathered afterwards -- checked on CPU
with two gloo ranks against the unsharded oracle -- and the host side of the
decode step's fused Q + latent projection weight."""

import multiprocessing as mp
import os

import numpy as np
import pytest

from llms_b200.mla import batch_shard


@pytest.mark.parametrize("B", [0, 1, 5, 8, 32, 33])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_batch_shards_partition_the_batch(B, world):
    rows = [list(batch_shard(B, world, r)) for r in range(world)]
    assert sum(rows, []) == list(range(B))  # disjoint, ordered, complete
    sizes = [len(x) for x in rows]
    assert max(sizes) - min(sizes) <= 1  # balanced


def test_batch_shard_rejects_bad_requests():
    with pytest.raises(ValueError):
        batch_shard(4, 0, 0)
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


def _mla_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from oracle import inputs as I
    from oracle import reference_math as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, L, dims = 5, 40, dict(H=8, KV=2, D=32, DR=8, R=24)
    d = I.cfg4(B, L, seed=9, **dims)
    inv = O.mla_inv_freq(dims["D"], dims["DR"], 1e6)
    rows = list(batch_shard(B, world, rank))
    mine = O.mla_decode(d["q"][rows], d["c_kv"][rows], d["k_rope_pre"][rows], d["w_uk"], d["w_uv"], d["k_norm_w"],
                        1e-6, inv, L)  # this rank streams only its own rows
    parts = [None] * world
    dist.all_gather_object(parts, mine)
    if rank == 0:
        full = O.mla_decode(d["q"], d["c_kv"], d["k_rope_pre"], d["w_uk"], d["w_uv"], d["k_norm_w"], 1e-6, inv, L)
        out.put(float(np.abs(np.concatenate(parts, 0) - full).max()))
    dist.destroy_process_group()


def test_batch_sharded_decode_gathers_to_full_output_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 1000
    procs = [ctx.Process(target=_mla_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-9


def test_q_latent_weight_is_one_buffer_of_views():
    """The decode step's fused Q + latent projection: q, dkv and kr weights
    become row views of one stacked buffer (no second copy), state dicts keep
    their keys, and the buffer follows in-place loads."""
    import torch
    from llms_b200.mla import B200MLAttention
    torch.manual_seed(0)
    m = B200MLAttention(hidden_size=64, num_heads=4, num_kv_heads=2, head_dim=16, rms_eps=1e-6, rank=32,
                        d_rope=8, max_position_embeddings=16, rope_theta=1e4)
    x = torch.zeros(1, 1, 64)
    ref = torch.cat([m.q.weight, m.dkv.weight, m.kr.weight]).detach().clone()
    W = m._q_latent_weight(x)
    assert W.shape == (64 + 32 + 16, 64) and torch.equal(W, ref)
    assert m.q.weight.data_ptr() == W.data_ptr()
    assert m.dkv.weight.data_ptr() == W[64:].data_ptr() and m.kr.weight.data_ptr() == W[96:].data_ptr()
    assert m._q_latent_weight(x) is W
    sd = {k: torch.randn_like(v) for k, v in m.state_dict().items()}
    m.load_state_dict(sd)
    assert torch.equal(W[:64], sd["q.weight"]) and torch.equal(W[96:], sd["kr.weight"])
    m.double()  # replaces the parameters' storage: rebuilt for float64 inputs
    assert m._q_latent_weight(x) is None
    W2 = m._q_latent_weight(x.double())
    assert W2.dtype == torch.float64 and m.dkv.weight.data_ptr() == W2[64:].data_ptr()


@pytest.mark.parametrize("B", [1, 2, 3, 8, 32])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_decode_shards_cover_every_row_and_group_once(B, world):
    from llms_b200.mla import decode_shard
    KV = 8
    seen = np.zeros((B, KV), int)
    busy = 0
    for r in range(world):
        rows, groups = decode_shard(B, KV, world, r)
        for b in rows:
            for g in groups:
                seen[b, g] += 1
        busy += bool(len(rows) and len(groups))
    assert (seen == 1).all()
    if B < world:  # fewer rows than GPUs: the group split keeps (nearly) every GPU busy
        assert busy >= min(world, B * KV) - (world % B if B > 1 else 0)


def _group_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from llms_b200.mla import decode_shard
    from oracle import inputs as I
    from oracle import reference_math as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, L, dims = 1, 40, dict(H=8, KV=4, D=32, DR=8, R=24)
    d = I.cfg4(B, L, seed=9, **dims)
    inv = O.mla_inv_freq(dims["D"], dims["DR"], 1e6)
    rows, groups = decode_shard(B, dims["KV"], world, rank)
    hpg = dims["H"] // dims["KV"]
    g0, g1 = groups.start, groups.stop
    # this rank reads its rows' whole latent, but only its groups' keys and heads
    mine = O.mla_decode(d["q"][list(rows)][:, g0 * hpg:g1 * hpg], d["c_kv"][list(rows)],
                        d["k_rope_pre"][list(rows)][:, :, g0:g1], d["w_uk"][g0:g1], d["w_uv"][g0:g1],
                        d["k_norm_w"], 1e-6, inv, L)
    parts = [None] * world
    dist.all_gather_object(parts, (list(rows), (g0, g1), mine))
    if rank == 0:
        full = O.mla_decode(d["q"], d["c_kv"], d["k_rope_pre"], d["w_uk"], d["w_uv"], d["k_norm_w"], 1e-6, inv, L)
        got = np.full_like(full, np.nan)
        for rws, (a, b), m in parts:
            if rws and b > a:
                got[rws, a * hpg:b * hpg] = m
        out.put(float(np.abs(got - full).max()))
    dist.destroy_process_group()


def test_group_sharded_decode_gathers_to_full_output_gloo():
    """B = 1 on two ranks: each rank serves half the KV groups' heads."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 1000
    procs = [ctx.Process(target=_group_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-9
