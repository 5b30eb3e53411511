"""GPU parity of the ``o`` / ``down`` projections (``b200mm_linear``,
``b200mm_linear_w8``) vs the oracle, at the Qwen3-4B shapes over the decode,
small-batch and prefill kernel families, and of the module swap in a decode
step."""

import numpy as np
import pytest
import torch

from oracle import inputs as I
from oracle import reference_math as O
from tests.conftest import bf16_check
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import llms_b200.kernels  # noqa: F401


def _rows(M, n=48, seed=0):
    if M <= n:
        return np.arange(M)
    return np.sort(np.random.default_rng(seed).choice(M, n, replace=False))


@pytest.mark.parametrize("which", ["o", "down"])
@pytest.mark.parametrize("M", [1, 2, 4, 7, 16, 40, 64, 129, 2048])
def test_linear_bf16(which, M):
    from llms_b200.kernels import b200_linear
    x, w = I.o_down(M, which)
    y = b200_linear(dev(x), dev(w))
    assert y.shape == (M, 2560) and y.dtype == torch.bfloat16
    r = _rows(M)
    bf16_check(host(y)[r], O.linear(x[r], w))


@pytest.mark.parametrize("M", [1, 3, 8])
def test_linear_fp16_and_fp32(M):
    from llms_b200.kernels import b200_linear
    x, w = I.o_down(M, "o")
    y16 = b200_linear(dev(x, torch.float16), dev(w, torch.float16))
    bf16_check(host(y16), O.linear(x, w))
    y32 = b200_linear(dev(x, torch.float32), dev(w, torch.float32))
    np.testing.assert_allclose(host(y32), O.linear(x, w), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("which", ["o", "down"])
@pytest.mark.parametrize("M", [1, 5, 32, 300])
def test_linear_int8(which, M):
    from llms_b200.kernels import int8_linear, quantize_per_row
    x, w = I.o_down(M, which)
    q, s = quantize_per_row(torch.from_numpy(w))
    y = int8_linear(dev(x), q.cuda(), s.cuda())
    r = _rows(M)
    bf16_check(host(y)[r], O.linear(x[r], O.dequant(q.numpy(), s.numpy())))


def test_linear_strided_and_3d():
    from llms_b200.kernels import b200_linear
    x, w = I.o_down(6, "o")
    xb = torch.zeros(6, 4096 + 64, dtype=torch.bfloat16, device="cuda")
    xb[:, :4096] = dev(x)
    y = b200_linear(xb[:, :4096].view(2, 3, 4096), dev(w))
    assert y.shape == (2, 3, 2560)
    bf16_check(host(y).reshape(6, 2560), O.linear(x, w))


def test_linear_rejects_bad_args():
    from llms_b200.kernels import b200_linear, int8_linear
    x = torch.zeros(2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        b200_linear(x, torch.zeros(8, 32, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        b200_linear(x, torch.zeros(8, 64, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        int8_linear(x, torch.zeros(8, 64, dtype=torch.int8, device="cuda"),
                    torch.ones(7, device="cuda"))


def test_swap_o_down_in_decode_step():
    """The eager engine block vs the same block after apply_triton_kernels +
    apply_linear_kernels: same weights, one decode token, parity of the
    block output."""
    from llms_b200.kernels import B200Linear, apply_linear_kernels, apply_triton_kernels
    from llms_b200.qwen3 import QWEN3_4B, Qwen3Model
    import dataclasses
    shape = dataclasses.replace(QWEN3_4B, num_hidden_layers=2, vocab_size=512)
    torch.manual_seed(0)
    m = Qwen3Model(shape).to("cuda", torch.bfloat16).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.02)
    ids = torch.randint(0, 512, (1, 5), device="cuda")
    with torch.inference_mode():
        c0 = m.alloc_cache(8)
        ref = m(ids, c0, start_pos=0).float()
        apply_triton_kernels(m)
        apply_linear_kernels(m)
        assert isinstance(m.layers[0].attn.o, B200Linear) and isinstance(m.layers[1].ffn.down, B200Linear)
        c1 = m.alloc_cache(8)
        out = m(ids, c1, start_pos=0).float()
    bf16_check(out.cpu().numpy(), ref.cpu().numpy(), max_abs=5e-2, rel_l2=2e-2)
