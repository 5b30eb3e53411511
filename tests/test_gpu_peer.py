"""b200mm_peer_gather on two GPUs: the peer-memory all-gather of the
column-sharded decode step against NCCL's all-gather on the same blocks, and
the sharded Qwen3-8B-shaped step with peer gathers -- at batch 1 and 4 fused
into the projection kernels (b200mm_*_peer), at batch 16 partly -- against the same
step with NCCL gathers (the arithmetic is the same, so the logits must be
identical).
One process per GPU; skipped with fewer than two GPUs."""

import multiprocessing as mp
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _expected(blocks, parts, world):
    """NCCL-free layout: part j of every rank together, rank order."""
    cols, start = [], 0
    for w in parts:
        for r in range(world):
            cols.append(blocks[r][:, start:start + w])
        start += w
    return torch.cat(cols, dim=1)


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    res = {}
    try:
        from llms_b200.peer import PeerGather
        ctx = PeerGather(16 << 20)
        for name, parts, rows in (("qkv16", (256, 64, 64), 5), ("odd2", (3, 5, 7), 3), ("one", (1216,), 64)):
            c = sum(parts)
            site = ctx.site(64, world * c, torch.bfloat16)
            for call in range(2):  # two calls in a row: the flags advance
                g = torch.Generator(device="cuda").manual_seed(100 * call + rank)
                y = torch.randn(rows, c, device="cuda", generator=g).to(torch.bfloat16)
                got = site.gather(y, parts).clone()
                blocks = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(blocks, y)
                res[f"{name}_{call}"] = bool(torch.equal(got, _expected(blocks, parts, world)))
        # inside a CUDA graph, replayed with new inputs
        site = ctx.site(16, world * 512, torch.bfloat16)
        y = torch.zeros(16, 512, device="cuda", dtype=torch.bfloat16)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            site.gather(y)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gy = site.gather(y)
        for call in range(3):
            y.copy_(torch.full((16, 512), float(10 * rank + call), device="cuda"))
            graph.replay()
            torch.cuda.synchronize()
            want = torch.cat([torch.full((16, 512), float(10 * r + call), device="cuda") for r in range(world)], 1)
            res[f"graph_{call}"] = bool(torch.equal(gy.float(), want))
            # a peer's next gather writes this site again: read it first
            dist.barrier()
        res["status"] = ctx.status()

        # the sharded 8B-shaped step (2 layers, small vocabulary): peer vs NCCL gathers
        from llms_b200.kernels import apply_decode_attn, apply_linear_kernels
        from llms_b200.qwen3 import QWEN3_8B, synthetic_int8_model
        from llms_b200.shard import peer_bytes, shard_decode_model
        import dataclasses
        shape = dataclasses.replace(QWEN3_8B, num_hidden_layers=2, vocab_size=4096)
        logits = {}
        for mode in ("nccl", "peer"):
            model = synthetic_int8_model(shape, seed=4)
            apply_linear_kernels(model, lm_head=True)
            apply_decode_attn(model)
            peer = PeerGather(peer_bytes(model, 16)) if mode == "peer" else None
            shard_decode_model(model, rank, world, peer=peer, max_rows=16)
            for B in (1, 4, 16):  # 1, 4: every projection fused with its gather; 16: int8 fused, bf16 + b200mm_peer_gather
                g = torch.Generator(device="cuda").manual_seed(5)
                ids = torch.randint(0, shape.vocab_size, (B, 8), device="cuda", generator=g)
                nxt = torch.randint(0, shape.vocab_size, (B, 1), device="cuda", generator=g)
                with torch.inference_mode():
                    cache = model.alloc_cache(16, max_batch=B)
                    model(ids, cache, start_pos=0)  # prefill: 8 B rows, the NCCL fallback above 16
                    for step in range(2):
                        logits[(mode, B, step)] = model(nxt, cache, start_pos=8 + step)[:, -1].float().cpu()
            if peer is not None:
                res["model_status"] = peer.status()
            del model, peer
        for B in (1, 4, 16):
            for step in range(2):
                res[f"model_equal_b{B}_{step}"] = bool(torch.equal(logits[("nccl", B, step)],
                                                                   logits[("peer", B, step)]))
        out.put((rank, res))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        out.put((rank, {"error": f"{type(e).__name__}: {e}"}))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs (one process per GPU)")
def test_peer_gather_matches_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(WORLD):
        res = results[r]
        assert "error" not in res, res
        assert res.pop("status") == 0 and res.pop("model_status") == 0, res
        assert all(res.values()), res
