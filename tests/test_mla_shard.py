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
def test_decode_shards_cover_every_row_and_token_once(B, world):
    from llms_b200.mla import decode_shard
    L = 1000
    seen = np.zeros((B, L), int)
    for r in range(world):
        rows, toks = decode_shard(B, L, world, r)
        seen[rows.start:rows.stop, toks.start:toks.stop] += 1
        if B < world:  # fewer rows than GPUs: every GPU streams a slice of every row
            assert len(rows) == B and len(toks) > 0
    assert (seen == 1).all()


def _partial(d, rows, toks, inv, L):
    """Float64 restatement of one context range's partial decode: the softmax
    of the range's tokens (max m, sum s) and the latent they mix (av)."""
    from oracle import reference_math as O
    q = np.asarray(d["q"][rows], np.float64)
    c = np.asarray(d["c_kv"][rows], np.float64)
    kr = np.asarray(d["k_rope_pre"][rows], np.float64)
    B, H, D = q.shape
    KV, DN, R = d["w_uk"].shape
    DR = D - DN
    k_nope = np.einsum("blr,gnr->blgn", c[:, :L], np.asarray(d["w_uk"], np.float64))
    k = O.rms_norm(np.concatenate([k_nope, kr[:, :L]], -1), d["k_norm_w"], 1e-6)
    cq, sq = O.rope_cos_sin(np.array([L - 1]), inv)
    ck, sk = O.rope_cos_sin(np.arange(L), inv)
    qr = q[..., DN:]
    q = np.concatenate([q[..., :DN], qr * cq[0] + O.rotate_half(qr) * sq[0]], -1)
    krr = k[..., DN:] * ck[None, :, None] + O.rotate_half(k[..., DN:]) * sk[None, :, None]
    k = np.repeat(np.concatenate([k[..., :DN], krr], -1), H // KV, axis=2)[:, toks.start:toks.stop]
    s = np.einsum("bhd,blhd->bhl", q, k) * D ** -0.5
    m = s.max(-1)
    p = np.exp(s - m[..., None])
    av = np.einsum("bhl,blr->bhr", p, c[:, toks.start:toks.stop]) / p.sum(-1)[..., None]
    return m, p.sum(-1), av


def _context_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from llms_b200.mla import decode_shard
    from oracle import inputs as I
    from oracle import reference_math as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, L, dims = 1, 40, dict(H=8, KV=2, D=32, DR=8, R=24)
    d = I.cfg4(B, L, seed=9, **dims)
    inv = O.mla_inv_freq(dims["D"], dims["DR"], 1e6)
    rows, toks = decode_shard(B, L, world, rank)
    mine = _partial(d, list(rows), toks, inv, L)  # this rank streams only its token slice
    parts = [None] * world
    dist.all_gather_object(parts, mine)  # the one exchange: B x H x (R + 2) numbers per rank
    if rank == 0:
        M = np.max([m for m, _, _ in parts], axis=0)
        wts = [s * np.exp(m - M) for m, s, _ in parts]
        av = sum(w[..., None] * a for w, (_, _, a) in zip(wts, parts)) / sum(wts)[..., None]
        g_of = np.arange(dims["H"]) // (dims["H"] // dims["KV"])
        got = np.einsum("bhr,hdr->bhd", av, np.asarray(d["w_uv"], np.float64)[g_of])
        full = O.mla_decode(d["q"], d["c_kv"], d["k_rope_pre"], d["w_uk"], d["w_uv"], d["k_norm_w"], 1e-6, inv, L)
        out.put(float(np.abs(got - full).max()))
    dist.destroy_process_group()


def test_context_split_decode_merges_to_full_output_gloo():
    """B = 1 on two ranks: each rank takes half the context; the merged
    partials equal the unsharded decode."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 1000
    procs = [ctx.Process(target=_context_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-9
