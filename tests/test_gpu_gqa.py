"""GPU parity of the GQA decode attention op (``b200mm_gqa_decode`` through
``llms_b200.kernels.b200_decode_attn``) vs the oracle, on the reference's
golden cases and on Qwen3 shapes with ragged, long and strided caches."""

import numpy as np
import pytest
import torch

from oracle import reference_math as O
from tests.conftest import bf16_check
from tests.gpu_util import dev, force_generic, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import llms_b200.kernels  # noqa: F401


def _rounded(a, dtype):
    return host(dev(a, dtype))


def _run(q, k, v, scale, dtype=torch.bfloat16):
    from llms_b200.kernels import b200_decode_attn
    out = b200_decode_attn(dev(q, dtype)[:, :, None], dev(k, dtype), dev(v, dtype), scale=scale)
    assert out.shape == (q.shape[0], q.shape[1], 1, q.shape[2]) and out.dtype == dtype
    return host(out[:, :, 0])


@pytest.mark.parametrize("name", ["gqa_b2_h8_kv2_d128_l38", "gqa_b3_h12_kv4_d64_l70", "gqa_b1_h4_kv4_d32_l5"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_golden(golden, name, dtype):
    g = lambda k: golden[f"{name}__{k}"]
    q, k, v, scale = g("q"), g("k"), g("v"), float(g("scale")[0])
    out = _run(q, k, v, scale, dtype)
    if dtype == torch.float32:
        np.testing.assert_allclose(out, g("out"), rtol=1e-4, atol=1e-5)
    else:
        qr, kr, vr = (_rounded(a, dtype) for a in (q, k, v))
        bf16_check(out, O.gqa_decode(qr, kr, vr, scale))


def _case(B, H, KV, D, L, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    k = rng.standard_normal((B, KV, L, D), dtype=np.float32)
    v = rng.standard_normal((B, KV, L, D), dtype=np.float32)
    return q, k, v


@pytest.mark.parametrize("L", [1, 2, 63, 64, 65, 129, 1000])
@pytest.mark.parametrize("B", [1, 3])
def test_qwen3_shape_ragged(B, L):
    q, k, v = _case(B, 32, 8, 128, L, seed=L)
    out = _run(q, k, v, 128 ** -0.5)
    qr, kr, vr = (_rounded(a, torch.bfloat16) for a in (q, k, v))
    bf16_check(out, O.gqa_decode(qr, kr, vr, 128 ** -0.5))


@pytest.mark.parametrize("H,KV,D", [(8, 8, 128), (16, 1, 128), (32, 8, 64), (12, 4, 64), (20, 4, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_groups_and_dims(H, KV, D, dtype):
    q, k, v = _case(2, H, KV, D, 300, seed=H + D)
    out = _run(q, k, v, D ** -0.5, dtype)
    qr, kr, vr = (_rounded(a, dtype) for a in (q, k, v))
    bf16_check(out, O.gqa_decode(qr, kr, vr, D ** -0.5))


def test_cache_views_with_garbage_past_L():
    """The op reads views of a larger cache (max batch, max length): rows past
    L hold NaN and must not leak into the result."""
    from llms_b200.kernels import b200_decode_attn
    B, H, KV, D, L, S = 3, 32, 8, 128, 77, 256
    q, k, v = _case(B, H, KV, D, L, seed=5)
    kc = torch.full((B + 2, KV, S, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    vc = torch.full((B + 2, KV, S, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    kc[:B, :, :L] = dev(k)
    vc[:B, :, :L] = dev(v)
    out = b200_decode_attn(dev(q)[:, :, None], kc[:B, :, :L], vc[:B, :, :L], scale=D ** -0.5)
    qr, kr, vr = (_rounded(a, torch.bfloat16) for a in (q, k, v))
    assert torch.isfinite(out).all()
    bf16_check(host(out[:, :, 0]), O.gqa_decode(qr, kr, vr, D ** -0.5))


@pytest.mark.parametrize("B,L", [(8, 32768), (32, 4096)])
def test_long_context_vs_torch_fp32(B, L):
    """Long caches: against the engine's own expression (repeat_interleave +
    SDPA) in fp32 on the device."""
    from llms_b200.kernels import b200_decode_attn
    g = torch.Generator(device="cuda").manual_seed(B)
    q = torch.randn(B, 32, 1, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, 8, L, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, 8, L, 128, device="cuda", generator=g).bfloat16()
    out = b200_decode_attn(q, k, v, scale=128 ** -0.5)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(4, dim=1), v.float().repeat_interleave(4, dim=1))
    bf16_check(out.float().cpu().numpy(), ref.cpu().numpy())


def test_generic_path_matches_split():
    q, k, v = _case(2, 32, 8, 128, 500, seed=9)
    fast = _run(q, k, v, 128 ** -0.5)
    with force_generic():
        slow = _run(q, k, v, 128 ** -0.5)
    bf16_check(fast, slow.astype(np.float64))


def test_rejects_bad_args():
    from llms_b200.kernels import b200_decode_attn
    q = torch.zeros(2, 8, 1, 64, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(2, 3, 5, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        b200_decode_attn(q, k, k, scale=0.1)  # 8 heads over 3 KV heads
    with pytest.raises(ValueError):
        b200_decode_attn(q, k[:, :2].float(), k[:, :2].float(), scale=0.1)


def test_decode_seam_in_model():
    """apply_decode_attn on a Qwen3-shaped model (2 layers): decode steps
    through the op agree with the default SDPA path."""
    import dataclasses
    from llms_b200.kernels import apply_decode_attn, apply_triton_kernels, b200_decode_attn
    from llms_b200.qwen3 import QWEN3_4B, Qwen3Model
    shape = dataclasses.replace(QWEN3_4B, num_hidden_layers=2, vocab_size=512)
    torch.manual_seed(0)
    m = Qwen3Model(shape).to("cuda", torch.bfloat16).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.02)
    ids = torch.randint(0, 512, (2, 40), device="cuda")
    with torch.inference_mode():
        for swap in (False, True):
            if swap:
                apply_triton_kernels(m)
                apply_decode_attn(m)
                assert m.layers[0].attn.decode_attn_op is b200_decode_attn
            c = m.alloc_cache(48, max_batch=2)
            m(ids, c, start_pos=0)
            outs = [m(ids[:, i:i + 1], c, start_pos=40 + i).float() for i in range(3)]
            if not swap:
                ref = outs
    for a, b in zip(outs, ref):
        bf16_check(a.cpu().numpy(), b.cpu().numpy(), max_abs=5e-2, rel_l2=2e-2)


def test_workspace_reuse_across_shapes():
    """Calls of different shapes share one workspace per stream: every call
    must leave the flag words clean for the next (no per-call memset)."""
    for B, L in ((2, 100), (4, 5000), (2, 100), (1, 33), (4, 5000)):
        q, k, v = _case(B, 32, 8, 128, L, seed=B * L)
        out = _run(q, k, v, 128 ** -0.5)
        qr, kr, vr = (_rounded(a, torch.bfloat16) for a in (q, k, v))
        bf16_check(out, O.gqa_decode(qr, kr, vr, 128 ** -0.5))
