"""Qwen3-8B-shaped int8 decode step: the model with the
int8 fused projections agrees with the same model run in fp32 with
dequantised weights, and its greedy next token matches wherever the fp32
top-2 gap exceeds the bf16 noise floor."""

import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model4():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200.qwen3 import QWEN3_8B, synthetic_int8_model
    shape = dataclasses.replace(QWEN3_8B, num_hidden_layers=4, max_position_embeddings=256)
    return synthetic_int8_model(shape, seed=4)


@pytest.mark.parametrize("B", [1, 16, 64])
def test_int8_decode_step_matches_fp32_dequant(model4, B):
    from llms_b200.qwen3 import greedy
    m = model4
    g = torch.Generator(device="cuda").manual_seed(B)
    P = 12
    prompt = torch.randint(0, m.shape.vocab_size, (B, P), generator=g, device="cuda")
    nxt = torch.randint(0, m.shape.vocab_size, (B, 1), generator=g, device="cuda")
    with torch.inference_mode():
        cache = m.alloc_cache(P + 4, max_batch=B)
        m(prompt, cache, start_pos=0)
        logits = m(nxt, cache, start_pos=P)[:, -1].float()
        ref_cache = m.alloc_cache(P + 4, max_batch=B, dtype=torch.float32)
        m.forward_fp32_dequant(prompt, ref_cache, 0)
        ref = m.forward_fp32_dequant(nxt, ref_cache, P)[:, -1]
    err = (logits - ref).abs().max().item()
    scale = ref.abs().max().item()
    rel = ((logits - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, f"logits rel-L2 {rel:.3e} (max abs {err:.3e}, |ref| max {scale:.3e})"
    top2 = ref.topk(2, dim=-1).values
    gap = top2[:, 0] - top2[:, 1]
    decided = gap > 4 * err  # rows whose argmax is not within the bf16 noise floor
    ours, theirs = greedy(logits), greedy(ref)
    assert decided.any(), "every row is a near-tie; widen the test"
    assert torch.equal(ours[decided], theirs[decided]), (
        f"argmax differs on decided rows: {(ours != theirs)[decided].sum().item()} of {decided.sum().item()}")


def test_swap_kernels_on_eager_model():
    """apply_int8_kernels on the eager model: the int8 model's output equals an
    eager model holding the dequantised weights."""
    from llms_b200.kernels import apply_int8_kernels, dequantize_per_row
    from llms_b200.qwen3 import Qwen3Model, Qwen3Shape
    shape = Qwen3Shape(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=512, max_position_embeddings=64)
    torch.manual_seed(0)
    m = Qwen3Model(shape).cuda().to(torch.bfloat16).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05)
    ids = torch.randint(0, 512, (2, 6), device="cuda")
    with torch.inference_mode():
        eager = m(ids, m.alloc_cache(16, max_batch=2), start_pos=0).float()
        apply_int8_kernels(m)
        ref = Qwen3Model(shape).cuda().to(torch.bfloat16).eval()
        ref.load_state_dict({k: v for k, v in m.state_dict().items() if k in ref.state_dict()}, strict=False)
        for rb, mb in zip(ref.layers, m.layers):
            W = dequantize_per_row(mb.attn.q_qkv, mb.attn.s_qkv).to(torch.bfloat16)
            rb.attn.q.weight.copy_(W[:256]); rb.attn.k.weight.copy_(W[256:384]); rb.attn.v.weight.copy_(W[384:])
            rb.ffn.gate.weight.copy_(dequantize_per_row(mb.ffn.qg, mb.ffn.sg).to(torch.bfloat16))
            rb.ffn.up.weight.copy_(dequantize_per_row(mb.ffn.qu, mb.ffn.su).to(torch.bfloat16))
        r = ref(ids, ref.alloc_cache(16, max_batch=2), start_pos=0).float()
        q = m(ids, m.alloc_cache(16, max_batch=2), start_pos=0).float()
    assert ((q - r).norm() / r.norm()).item() < 2e-2
    assert ((q - eager).norm() / eager.norm()).item() < 0.2  # int8 rounding of the weights


def test_graphed_decode_step_matches_eager():
    """GraphedDecodeStep: one CUDA graph of the whole decode step, replayed at
    successive positions, against eager decode steps on a separate cache."""
    import dataclasses
    from llms_b200.kernels import apply_linear_kernels, apply_triton_kernels
    from llms_b200.qwen3 import QWEN3_4B, GraphedDecodeStep, Qwen3Model
    from tests.conftest import bf16_check
    shape = dataclasses.replace(QWEN3_4B, num_hidden_layers=2, vocab_size=512)
    torch.manual_seed(0)
    m = Qwen3Model(shape).to("cuda", torch.bfloat16).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.02)
    apply_triton_kernels(m)
    apply_linear_kernels(m)
    ids = torch.randint(0, 512, (2, 20), device="cuda")
    nxt = torch.randint(0, 512, (3, 2, 1), device="cuda")
    with torch.inference_mode():
        ca, cb = m.alloc_cache(64, max_batch=2), m.alloc_cache(64, max_batch=2)
        m(ids, ca, start_pos=0)
        m(ids, cb, start_pos=0)
        step = GraphedDecodeStep(m, cb, batch=2)
        for i in range(3):
            ref = m(nxt[i], ca, start_pos=20 + i).float()
            got = step(nxt[i], 20 + i).float()
            bf16_check(got.cpu().numpy(), ref.cpu().numpy(), max_abs=5e-2, rel_l2=2e-2)
    assert cb.cur_len == 23


@pytest.fixture(scope="module")
def golden_model():
    """Config 5 at 2 layers / 4096 vocabulary on the device: the weights the
    reference engine ran in tests/golden/make_golden.py."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200.qwen3 import QWEN3_8B, dequantized_dense_model, int8_model_from_state
    from oracle import inputs as I
    shape = dataclasses.replace(QWEN3_8B, num_hidden_layers=2, vocab_size=4096, max_position_embeddings=64)
    m = int8_model_from_state(I.cfg5_model(layers=2, vocab=4096), shape)
    return m, dequantized_dense_model(m)


def _decode_logits(model, ids, nxt):
    with torch.inference_mode():
        cache = model.alloc_cache(ids.shape[1] + 2, max_batch=ids.shape[0])
        model(ids, cache, start_pos=0)
        return model(nxt, cache, start_pos=ids.shape[1])[:, -1].float().cpu()


def test_int8_step_matches_reference_engine(golden, golden_model):
    """The int8 decode step (b200mm int8 QKV / gate-up, b200mm_linear o / down)
    against the reference engine's fp32 logits (golden), next to the reference
    engine's own bf16 arithmetic on the same weights (dequantised bf16
    nn.Linear, torch kernels).  Bars: logits rel-L2 <= 1.25x the reference
    bf16 path's; greedy argmax equal on every row whose fp32 top-2 gap exceeds
    the reference bf16 path's largest logit error on that row, and at least
    half the rows decided."""
    import numpy as np
    from llms_b200.kernels import apply_linear_kernels
    from llms_b200.qwen3 import greedy
    from oracle import inputs as I
    m, dense = golden_model
    ids, nxt = (torch.from_numpy(a).cuda() for a in I.cfg5_tokens(16, 6, 4096))
    ref = torch.from_numpy(golden["qwen3_8b_int8_l2__logits"])
    base = _decode_logits(dense, ids, nxt)
    apply_linear_kernels(m)
    ours = _decode_logits(m, ids, nxt)
    rel = lambda a: ((a - ref).norm() / ref.norm()).item()
    assert rel(ours) <= 1.25 * rel(base) + 1e-4, f"rel-L2 ours {rel(ours):.3e}, reference bf16 path {rel(base):.3e}"
    top2 = ref.topk(2, dim=-1).values
    decided = (top2[:, 0] - top2[:, 1]) > (base - ref).abs().amax(-1)
    assert decided.sum().item() >= ref.shape[0] // 2, f"only {decided.sum().item()} of {ref.shape[0]} rows decided"
    want = torch.from_numpy(golden["qwen3_8b_int8_l2__argmax"].astype(np.int64))
    got = greedy(ours)
    assert torch.equal(got[decided], want[decided]), f"argmax differs on {(got != want)[decided].sum().item()} rows"
