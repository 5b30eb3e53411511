"""GPU parity of the fused QKV / gate-up-SiLU / int8 kernels vs the oracle
(and the reference's golden outputs).  Calls go through the reference-facing
shim, which calls the C ABI."""

import numpy as np
import pytest
import torch

from oracle import inputs as I
from oracle import reference_math as O
from tests.conftest import bf16_check
from tests.gpu_util import dev, force_generic, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import llms_b200.kernels  # noqa: F401  (fails loudly if the library is missing)


def test_cfg1_fp32_gate_up_vs_golden(golden):
    from llms_b200.kernels import triton_fused_gate_up_silu
    x, wg, wu = I.cfg1()
    y = triton_fused_gate_up_silu(dev(x, torch.float32), dev(wg, torch.float32), dev(wu, torch.float32))
    assert y.dtype == torch.float32 and y.shape == (4, 3072)
    np.testing.assert_allclose(host(y), golden["cfg1_gate_up"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(host(y), O.gate_up_silu(x, wg, wu), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("M", [1, 4])
def test_cfg2_qkv_vs_golden(golden, M):
    from llms_b200.kernels import triton_fused_qkv
    x, w = I.cfg2(M)
    q, k, v = triton_fused_qkv(dev(x), dev(w), n_q=4096, n_k=1024)
    for name, t in (("q", q), ("k", k), ("v", v)):
        bf16_check(host(t), golden[f"cfg2_m{M}_{name}"])


@pytest.mark.parametrize("M", [1, 4])
def test_cfg3_gate_up_vs_golden(golden, M):
    from llms_b200.kernels import triton_fused_gate_up_silu
    x, wg, wu = I.cfg3(M)
    y = triton_fused_gate_up_silu(dev(x), dev(wg), dev(wu))
    bf16_check(host(y), golden[f"cfg3_m{M}_gate_up"])


def _rows_subset(M, n=48, seed=0):
    if M <= n:
        return np.arange(M)
    return np.sort(np.random.default_rng(seed).choice(M, n, replace=False))


@pytest.mark.parametrize("M", [1, 4, 16, 128, 2048])
def test_cfg2_qkv_all_m(M):
    from llms_b200.kernels import triton_fused_qkv
    x, w = I.cfg2(M)
    q, k, v = triton_fused_qkv(dev(x), dev(w), n_q=4096, n_k=1024)
    assert q.shape == (M, 4096) and k.shape == (M, 1024) and v.shape == (M, 1024)
    assert q.data_ptr() + 4096 * 2 == k.data_ptr()  # zero-copy split of one buffer
    rows = _rows_subset(M)
    eq, ek, ev = O.qkv(x[rows], w, 4096, 1024)
    for t, e in ((q, eq), (k, ek), (v, ev)):
        bf16_check(host(t)[rows], e)


@pytest.mark.parametrize("M", [1, 4, 16, 128, 2048])
def test_cfg3_gate_up_all_m(M):
    from llms_b200.kernels import triton_fused_gate_up_silu
    x, wg, wu = I.cfg3(M)
    y = triton_fused_gate_up_silu(dev(x), dev(wg), dev(wu))
    rows = _rows_subset(M)
    bf16_check(host(y)[rows], O.gate_up_silu(x[rows], wg, wu))


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 33])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gate_up_small_m_dtypes(M, dtype):
    from llms_b200.kernels import triton_fused_gate_up_silu
    rng = np.random.default_rng(M)
    x = rng.standard_normal((M, 512), dtype=np.float32)
    wg = rng.standard_normal((300, 512), dtype=np.float32) * 0.05
    wu = rng.standard_normal((300, 512), dtype=np.float32) * 0.05
    xd, wgd, wud = dev(x, dtype), dev(wg, dtype), dev(wu, dtype)
    y = triton_fused_gate_up_silu(xd, wgd, wud)
    assert y.dtype == dtype
    bf16_check(host(y), O.gate_up_silu(host(xd), host(wgd), host(wud)))


def test_non_pow2_N():
    """Reference tests/test_kernels_fused_ffn.py:155-177: N = 9700."""
    from llms_b200.kernels import triton_fused_gate_up_silu
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 2560), dtype=np.float32)
    wg = rng.standard_normal((9700, 2560), dtype=np.float32) * 0.02
    wu = rng.standard_normal((9700, 2560), dtype=np.float32) * 0.02
    xd, wgd, wud = dev(x), dev(wg), dev(wu)
    y = triton_fused_gate_up_silu(xd, wgd, wud)
    assert y.shape == (1, 9700)
    bf16_check(host(y), O.gate_up_silu(host(xd), host(wgd), host(wud)))


@pytest.mark.parametrize("M", [1, 5])
def test_qkv_odd_K(M):
    """Reference tests/test_kernels_fused_qkv.py:171-195: K = 2541 (rows not
    16-byte aligned, served by the general kernel)."""
    from llms_b200.kernels import triton_fused_qkv
    rng = np.random.default_rng(2)
    x = rng.standard_normal((M, 2541), dtype=np.float32)
    w = rng.standard_normal((4096 + 2048, 2541), dtype=np.float32) * 0.02
    xd, wd = dev(x), dev(w)
    q, k, v = triton_fused_qkv(xd, wd, n_q=4096, n_k=1024)
    e = O.qkv(host(xd), host(wd), 4096, 1024)
    for t, ee in zip((q, k, v), e):
        bf16_check(host(t), ee)


def test_leading_dims_and_strided_x():
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    rng = np.random.default_rng(3)
    big = dev(rng.standard_normal((2, 3, 128), dtype=np.float32))
    x = big[..., :64]                      # row stride 128, inner stride 1
    wg = dev(rng.standard_normal((128, 64), dtype=np.float32) * 0.1)
    wu = dev(rng.standard_normal((128, 64), dtype=np.float32) * 0.1)
    y = triton_fused_gate_up_silu(x, wg, wu)
    assert y.shape == (2, 3, 128)
    bf16_check(host(y), O.gate_up_silu(host(x), host(wg), host(wu)))
    w = dev(rng.standard_normal((32 + 32, 64), dtype=np.float32) * 0.1)
    q, k, v = triton_fused_qkv(x, w, n_q=32, n_k=16)
    assert q.shape == (2, 3, 32) and k.shape == (2, 3, 16) and v.shape == (2, 3, 16)
    xt = dev(rng.standard_normal((64, 6), dtype=np.float32)).t()  # inner stride != 1
    y2 = triton_fused_gate_up_silu(xt, wg, wu)
    bf16_check(host(y2), O.gate_up_silu(host(xt), host(wg), host(wu)))


def test_head_view_reshape():
    from llms_b200.kernels import triton_fused_qkv
    x = torch.randn(1, 5, 2560, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(6144, 2560, device="cuda", dtype=torch.bfloat16) * 0.02
    q, k, v = triton_fused_qkv(x, W, n_q=4096, n_k=1024)
    assert q.view(1, 5, 32, 128).shape == (1, 5, 32, 128)
    assert k.view(1, 5, 8, 128).shape == (1, 5, 8, 128)
    assert v.view(1, 5, 8, 128).shape == (1, 5, 8, 128)


def test_empty_batch():
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    x = torch.empty(0, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(96, 64, device="cuda", dtype=torch.bfloat16)
    assert triton_fused_gate_up_silu(x, w, w).shape == (0, 96)
    q, k, v = triton_fused_qkv(x, w, n_q=64, n_k=16)
    assert q.shape == (0, 64) and v.shape == (0, 16)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_generic_matches_fast(M):
    """The specialised kernels agree with the general tiled kernel."""
    from llms_b200.kernels import triton_fused_gate_up_silu
    x, wg, wu = I.cfg3(M)
    xd, wgd, wud = dev(x), dev(wg), dev(wu)
    fast = triton_fused_gate_up_silu(xd, wgd, wud)
    with force_generic():
        slow = triton_fused_gate_up_silu(xd, wgd, wud)
    bf16_check(host(fast), host(slow).astype(np.float64), max_abs=2e-2, rel_l2=5e-3)


@pytest.mark.parametrize("M", [1, 4])
def test_cfg5_int8_vs_golden(golden, M):
    from llms_b200.kernels import int8_fused_gate_up_silu, int8_fused_qkv
    lay = I.cfg5_layer(M=M)
    x = dev(lay["x"])
    to = lambda a: torch.from_numpy(a).cuda()
    q, k, v = int8_fused_qkv(x, to(lay["qkv_q"]), to(lay["qkv_s"]), n_q=4096, n_k=1024)
    bf16_check(np.concatenate([host(q), host(k), host(v)], -1), golden[f"cfg5_m{M}_qkv"])
    y = int8_fused_gate_up_silu(x, to(lay["gate_q"]), to(lay["gate_s"]), to(lay["up_q"]), to(lay["up_s"]))
    bf16_check(host(y), golden[f"cfg5_m{M}_gate_up"])


@pytest.mark.parametrize("M", [1, 16, 64])
def test_cfg5_int8_batches(M):
    from llms_b200.kernels import int8_fused_gate_up_silu, int8_fused_qkv
    lay = I.cfg5_layer(M=M)
    x = dev(lay["x"])
    to = lambda a: torch.from_numpy(a).cuda()
    rows = _rows_subset(M, 16)
    q, k, v = int8_fused_qkv(x, to(lay["qkv_q"]), to(lay["qkv_s"]), n_q=4096, n_k=1024)
    eq = O.qkv(lay["x"][rows], O.dequant(lay["qkv_q"], lay["qkv_s"]), 4096, 1024)
    for t, e in zip((q, k, v), eq):
        bf16_check(host(t)[rows], e)
    y = int8_fused_gate_up_silu(x, to(lay["gate_q"]), to(lay["gate_s"]), to(lay["up_q"]), to(lay["up_s"]))
    e = O.gate_up_silu(lay["x"][rows], O.dequant(lay["gate_q"], lay["gate_s"]), O.dequant(lay["up_q"], lay["up_s"]))
    bf16_check(host(y)[rows], e)


def test_modules_match_eager():
    """TritonFFN / TritonAttention projections equal the eager nn.Linear ones."""
    import torch.nn.functional as F
    from torch import nn
    from llms_b200.kernels import TritonFFN, triton_fused_qkv

    class FFN(nn.Module):
        def __init__(s):
            super().__init__()
            s.gate = nn.Linear(256, 512, bias=False)
            s.up = nn.Linear(256, 512, bias=False)
            s.down = nn.Linear(512, 256, bias=False)

        def forward(s, x):
            return s.down(F.silu(s.gate(x)) * s.up(x))

    torch.manual_seed(0)
    eager = FFN().cuda().to(torch.float32)
    fused = TritonFFN.from_eager(eager)
    assert fused.gate.weight is eager.gate.weight
    x = torch.randn(2, 3, 256, device="cuda")
    with torch.no_grad():
        torch.testing.assert_close(fused(x), eager(x), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M", [5, 7, 12, 24, 48, 64, 65, 100])
@pytest.mark.parametrize("gate", [False, True])
def test_mid_m_tensor_core_gemv(M, gate):
    """5 <= M <= 16 runs the mma.sync GEMV (K split over a 4-CTA cluster),
    17 <= M <= 64 the tcgen05 kernel with the weights on the MMA's M side,
    65 <= M < 128 the tcgen05 GEMM with a partly filled tile."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    rng = np.random.default_rng(M + 100 * gate)
    K, N = 2560, 1000  # N not a multiple of the 128-row group
    x = rng.standard_normal((M, K), dtype=np.float32)
    w0 = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    xd, w0d = dev(x), dev(w0)
    if gate:
        w1d = dev(rng.standard_normal((N, K), dtype=np.float32) * 0.02)
        y = triton_fused_gate_up_silu(xd, w0d, w1d)
        e = O.gate_up_silu(host(xd), host(w0d), host(w1d))
    else:
        q, k, v = triton_fused_qkv(xd, w0d, n_q=N - 200, n_k=100)
        y = torch.cat([q, k, v], -1)
        e = host(xd).astype(np.float64) @ host(w0d).astype(np.float64).T
    bf16_check(host(y), e)


@pytest.mark.parametrize("M", [2, 3, 5, 16, 33, 64])
def test_mid_m_int8_and_fp16(M):
    from llms_b200.kernels import int8_fused_gate_up_silu, int8_fused_qkv, triton_fused_qkv
    lay = I.cfg5_layer(M=M, seed=M)
    to = lambda a: torch.from_numpy(a[:1500]).cuda()
    x = dev(lay["x"])
    y = int8_fused_gate_up_silu(x, to(lay["gate_q"]), to(lay["gate_s"]), to(lay["up_q"]), to(lay["up_s"]))
    e = O.gate_up_silu(lay["x"], O.dequant(lay["gate_q"][:1500], lay["gate_s"][:1500]),
                       O.dequant(lay["up_q"][:1500], lay["up_s"][:1500]))
    bf16_check(host(y), e)
    q, k, v = int8_fused_qkv(x, to(lay["qkv_q"]), to(lay["qkv_s"]), n_q=1300, n_k=100)
    e = lay["x"].astype(np.float64) @ O.dequant(lay["qkv_q"][:1500], lay["qkv_s"][:1500]).T
    bf16_check(host(torch.cat([q, k, v], -1)), e)
    xh = dev(lay["x"], torch.float16)
    wh = dev(lay["qkv_q"][:768].astype(np.float32) * 0.01, torch.float16)
    q, k, v = triton_fused_qkv(xh, wh, n_q=512, n_k=128)
    e = host(xh).astype(np.float64) @ host(wh).astype(np.float64).T
    bf16_check(host(torch.cat([q, k, v], -1)), e)


@pytest.mark.parametrize("K", [2536, 1000])
def test_mid_m_k_tails(K):
    from llms_b200.kernels import triton_fused_gate_up_silu
    rng = np.random.default_rng(K)
    x = dev(rng.standard_normal((16, K), dtype=np.float32))
    wg = dev(rng.standard_normal((700, K), dtype=np.float32) * 0.03)
    wu = dev(rng.standard_normal((700, K), dtype=np.float32) * 0.03)
    y = triton_fused_gate_up_silu(x, wg, wu)
    bf16_check(host(y), O.gate_up_silu(host(x), host(wg), host(wu)))


@pytest.mark.parametrize("M,gate", [(129, False), (200, True), (256, False), (256, True)])
def test_tcgen05_partial_m_tiles(M, gate):
    """129 <= M <= 256: the tcgen05 GEMM with a partly filled second tile."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    rng = np.random.default_rng(M)
    K, N = 1536, 640
    xd = dev(rng.standard_normal((M, K), dtype=np.float32))
    w0d = dev(rng.standard_normal((N, K), dtype=np.float32) * 0.03)
    if gate:
        w1d = dev(rng.standard_normal((N, K), dtype=np.float32) * 0.03)
        bf16_check(host(triton_fused_gate_up_silu(xd, w0d, w1d)), O.gate_up_silu(host(xd), host(w0d), host(w1d)))
    else:
        q, k, v = triton_fused_qkv(xd, w0d, n_q=512, n_k=64)
        e = host(xd).astype(np.float64) @ host(w0d).astype(np.float64).T
        bf16_check(host(torch.cat([q, k, v], -1)), e)


@pytest.mark.parametrize("M", [100, 300, 2048])
def test_int8_prefill_m(M):
    """int8 weights at prefill sizes: several 256-row N tiles of activations."""
    from llms_b200.kernels import int8_fused_gate_up_silu, int8_fused_qkv
    lay = I.cfg5_layer(M=M, seed=M)
    rows = _rows_subset(M, 24)
    to = lambda a: torch.from_numpy(a[:1024]).cuda()
    x = dev(lay["x"])
    y = int8_fused_gate_up_silu(x, to(lay["gate_q"]), to(lay["gate_s"]), to(lay["up_q"]), to(lay["up_s"]))
    e = O.gate_up_silu(lay["x"][rows], O.dequant(lay["gate_q"][:1024], lay["gate_s"][:1024]),
                       O.dequant(lay["up_q"][:1024], lay["up_s"][:1024]))
    bf16_check(host(y)[rows], e)
    q, k, v = int8_fused_qkv(x, to(lay["qkv_q"]), to(lay["qkv_s"]), n_q=768, n_k=128)
    e = lay["x"][rows].astype(np.float64) @ O.dequant(lay["qkv_q"][:1024], lay["qkv_s"][:1024]).T
    bf16_check(host(torch.cat([q, k, v], -1))[rows], e)


@pytest.mark.parametrize("M,N,K", [(1, 96, 2560), (1, 768, 2560), (3, 1216, 4096), (2, 770, 2560), (1, 4000, 1024)])
@pytest.mark.parametrize("gate", [False, True])
def test_decode_column_shards(M, N, K, gate):
    """Decode on a column shard (down to N/8 of a layer, odd N, odd M)."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    rng = np.random.default_rng(N + K + M)
    xd = dev(rng.standard_normal((M, K), dtype=np.float32))
    w0d = dev(rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    if gate:
        w1d = dev(rng.standard_normal((N, K), dtype=np.float32) * 0.02)
        bf16_check(host(triton_fused_gate_up_silu(xd, w0d, w1d)), O.gate_up_silu(host(xd), host(w0d), host(w1d)))
    else:
        nk = N // 8
        q, k, v = triton_fused_qkv(xd, w0d, n_q=N - 2 * nk, n_k=nk)
        e = host(xd).astype(np.float64) @ host(w0d).astype(np.float64).T
        bf16_check(host(torch.cat([q, k, v], -1)), e)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_fp32_accumulation_meets_bare_bar(M):
    """The stated bar with no storage term: on bf16-representable inputs held
    in fp32 (so every product is exact), the fused projections' fp32 outputs
    -- the accumulation before any output rounding -- meet max-abs <= 2e-2 and
    rel-L2 <= 5e-3 against the float64 oracle at the Qwen3-4B shapes."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    x, w = I.cfg2(M)
    q, k, v = triton_fused_qkv(dev(x, torch.float32), dev(w, torch.float32), n_q=4096, n_k=1024)
    eq, ek, ev = O.qkv(x, w, 4096, 1024)
    bf16_check(host(torch.cat([q, k, v], -1)), np.concatenate([eq, ek, ev], -1), store_ulp=0.0)
    x, wg, wu = I.cfg3(M)
    y = triton_fused_gate_up_silu(dev(x, torch.float32), dev(wg, torch.float32), dev(wu, torch.float32))
    bf16_check(host(y), O.gate_up_silu(x, wg, wu), store_ulp=0.0)
