"""Host-side logic on CPU: module swaps (reference kernels/swap.py
semantics), int8 quantisation, and the column sharding used by the
multi-GPU bench (checked with two gloo ranks)."""

import os

import numpy as np
import torch
import torch.multiprocessing as mp


def tiny():
    from llms_b200.qwen3 import Qwen3Model, Qwen3Shape
    shape = Qwen3Shape(vocab_size=64, hidden_size=32, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=8, intermediate_size=48, max_position_embeddings=16)
    torch.manual_seed(0)
    return Qwen3Model(shape)


def test_apply_triton_kernels_swaps_and_is_idempotent():
    from llms_b200.kernels import TritonAttention, TritonFFN, apply_triton_kernels
    m = tiny()
    gate0 = m.layers[0].ffn.gate.weight
    q0, k0, v0 = m.layers[0].attn.q.weight, m.layers[0].attn.k.weight, m.layers[0].attn.v.weight
    apply_triton_kernels(m)
    assert all(isinstance(b.ffn, TritonFFN) and isinstance(b.attn, TritonAttention) for b in m.layers)
    assert m.layers[0].ffn.gate.weight is gate0  # shared, not copied
    assert torch.equal(m.layers[0].attn.W_qkv, torch.cat([q0, k0, v0], 0))
    first = [b.ffn for b in m.layers]
    apply_triton_kernels(m)
    assert all(a is b.ffn for a, b in zip(first, m.layers))


def test_apply_linear_kernels_swaps_o_and_down():
    from llms_b200.kernels import (B200Linear, Int8Linear, apply_linear_kernels, apply_triton_kernels,
                                   dequantize_per_row)
    m = tiny()
    o0, d0 = m.layers[0].attn.o.weight, m.layers[1].ffn.down.weight
    apply_triton_kernels(m)
    apply_linear_kernels(m)
    assert all(isinstance(b.attn.o, B200Linear) and isinstance(b.ffn.down, B200Linear) for b in m.layers)
    assert m.layers[0].attn.o.weight is o0 and m.layers[1].ffn.down.weight is d0
    first = [b.attn.o for b in m.layers]
    apply_linear_kernels(m)  # idempotent
    assert all(a is b.attn.o for a, b in zip(first, m.layers))
    sd = m.state_dict()
    assert "layers.0.attn.o.weight" in sd and "layers.1.ffn.down.weight" in sd

    m8 = tiny()
    d = m8.layers[0].ffn.down.weight.detach().clone()
    apply_linear_kernels(m8, int8=True, o=False)
    assert isinstance(m8.layers[0].ffn.down, Int8Linear) and isinstance(m8.layers[0].attn.o, torch.nn.Linear)
    lin = m8.layers[0].ffn.down
    assert lin.qweight.dtype == torch.int8 and lin.scale.shape == (d.shape[0],)
    err = (dequantize_per_row(lin.qweight, lin.scale) - d).abs()
    assert (err <= lin.scale[:, None] / 2 + 1e-7).all()


def test_linear_module_rejects_bias():
    import pytest
    from llms_b200.kernels import B200Linear, Int8Linear
    with pytest.raises(ValueError):
        B200Linear.from_linear(torch.nn.Linear(4, 4, bias=True))
    with pytest.raises(ValueError):
        Int8Linear.from_linear(torch.nn.Linear(4, 4, bias=True))


def test_apply_triton_kernels_flags():
    from llms_b200.kernels import TritonAttention, TritonFFN, apply_triton_kernels
    m = tiny()
    apply_triton_kernels(m, fused_ffn=False)
    assert not isinstance(m.layers[0].ffn, TritonFFN) and isinstance(m.layers[0].attn, TritonAttention)


def test_prewarm_no_op_without_kernel_modules():
    from llms_b200.kernels import prewarm_triton_kernels
    prewarm_triton_kernels(torch.nn.Sequential(torch.nn.Linear(4, 4)))


def test_quantize_per_row():
    from llms_b200.kernels import dequantize_per_row, quantize_per_row
    torch.manual_seed(1)
    W = torch.randn(37, 50)
    W[3] = 0
    q, s = quantize_per_row(W)
    assert q.dtype == torch.int8 and s.dtype == torch.float32 and q.abs().max() <= 127
    assert s[3] == 1 and (q[3] == 0).all()
    err = (dequantize_per_row(q, s) - W).abs()
    assert (err <= s[:, None] / 2 + 1e-7).all()  # round-to-nearest: half a step per row


def test_apply_int8_kernels_on_cpu_model():
    from llms_b200.kernels import Int8Attention, Int8FFN, apply_int8_kernels
    m = tiny()
    down0 = m.layers[1].ffn.down
    apply_int8_kernels(m)
    assert all(isinstance(b.ffn, Int8FFN) and isinstance(b.attn, Int8Attention) for b in m.layers)
    assert m.layers[1].ffn.down is down0
    assert m.layers[0].attn.q_qkv.shape == (32 + 2 * 16, 32)


def test_shard_plan_covers_every_row_once():
    import bench
    for world in (1, 2, 4, 8):
        rows = np.concatenate([bench.qkv_rows(r, world) for r in range(world)])
        assert sorted(rows.tolist()) == list(range(bench.NQ + 2 * bench.NK))
        cols = [bench.ffn_cols(r, world) for r in range(world)]
        assert cols[0][0] == 0 and cols[-1][1] == bench.INTER
        assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
        per = bench.qkv_rows(0, world)  # head-aligned: whole q heads + one k and one v block
        assert len(per) == (32 // world + 2 * (8 // world)) * bench.HEAD


def _gather_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 64, generator=g)
    W = torch.randn(bench.NQ + 2 * bench.NK, 64, generator=g)
    rows = torch.from_numpy(bench.qkv_rows(rank, world))
    part = x @ W[rows].T                      # this rank's column shard
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)
    if rank == 0:
        allrows = torch.cat([torch.from_numpy(bench.qkv_rows(r, world)) for r in range(world)])
        full = torch.empty(1, W.shape[0])
        full[:, allrows] = torch.cat(parts, -1)
        out.put(float((full - x @ W.T).abs().max()))
    dist.destroy_process_group()


def test_column_shards_gather_to_full_output_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-4


def test_forward_static_matches_forward_on_cpu():
    """The device-position decode step (what a CUDA graph replays at every
    position) gives the engine's decode result, step after step."""
    m = tiny().eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.2)
    ids = torch.randint(0, 64, (2, 6))
    with torch.no_grad():
        ca, cb = m.alloc_cache(12, max_batch=2), m.alloc_cache(12, max_batch=2)
        m(ids, ca, start_pos=0)
        m(ids, cb, start_pos=0)
        for step in range(4):
            nxt = torch.randint(0, 64, (2, 1))
            ref = m(nxt, ca, start_pos=6 + step)
            got = m.forward_static(nxt, cb, torch.tensor([6 + step]))
            torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(cb.k[1][:, :, :10], ca.k[1][:, :, :10])
