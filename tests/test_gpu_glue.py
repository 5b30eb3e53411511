"""GPU parity of the decode-step glue kernels (``b200mm_rmsnorm``,
``b200mm_qk_norm_rope``) against the engine's eager torch ops they replace:
RMSNorm (engine/attention.py:20-33), the residual add (engine/model.py:54-63),
q_norm / k_norm / apply_rope / the cache write (engine/attention.py:119-131).
The kernels keep the engine's rounding points, so results agree to within one
rounding step of the output dtype (the fp32 mean is summed in another order)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp_close(a, e, dtype):
    """|a - e| <= one rounding step of ``dtype`` at |e| (plus a tiny floor)."""
    eps = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10, torch.float32: 2.0 ** -20}[dtype]
    a, e = a.double(), e.double()
    bad = (a - e).abs() > eps * e.abs() + 1e-6
    assert not bad.any(), f"{int(bad.sum())} elements off; worst {float((a - e).abs().max()):.3e}"


def _eager_norm(x, w, eps):
    from llms_b200.kernels._eager import rms_norm
    return rms_norm(x, w, eps)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("M,N", [(1, 4096), (7, 2560), (64, 128), (3, 1024)])
def test_rmsnorm_matches_engine(dtype, M, N):
    from llms_b200.kernels.glue import rms_norm
    g = torch.Generator(device="cuda").manual_seed(M * N)
    x = (torch.randn(M, N, device="cuda", generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(N, device="cuda", generator=g)).to(dtype)
    _ulp_close(rms_norm(x, w, 1e-6), _eager_norm(x, w, 1e-6), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rmsnorm_residual_add(dtype):
    """h = cast(x + r) exactly as the engine's add; y = norm(h); 3-D inputs."""
    from llms_b200.kernels.glue import rms_norm
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4, 1, 4096, device="cuda", generator=g).to(dtype)
    r = torch.randn(4, 1, 4096, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(4096, device="cuda", generator=g)).to(dtype)
    h, y = rms_norm(x, w, 1e-6, residual=r)
    assert h.shape == x.shape and y.shape == x.shape
    assert torch.equal(h, x + r)
    _ulp_close(y, _eager_norm(x + r, w, 1e-6), dtype)


@pytest.mark.parametrize("D,H,KV", [(128, 32, 8), (64, 8, 2), (128, 4, 4)])
@pytest.mark.parametrize("device_pos", [False, True])
def test_qk_norm_rope_cache_matches_engine(D, H, KV, device_pos):
    from llms_b200.kernels._eager import RMSNorm, rope
    from llms_b200.kernels.glue import qk_norm_rope_cache
    from llms_b200.qwen3 import rope_tables
    dt = torch.bfloat16
    B, S, pos = 3, 40, 17
    g = torch.Generator(device="cuda").manual_seed(D + H)
    qkv = (torch.randn(B, 1, (H + 2 * KV) * D, device="cuda", generator=g) * 2).to(dt)
    qn, kn = RMSNorm(D).cuda().to(dt), RMSNorm(D).cuda().to(dt)
    with torch.no_grad():
        qn.weight.copy_(1 + 0.1 * torch.randn(D, device="cuda", generator=g))
        kn.weight.copy_(1 + 0.1 * torch.randn(D, device="cuda", generator=g))
    cos, sin = (t.cuda().to(dt) for t in rope_tables(D, 64, 1e6))
    kc = torch.full((B + 1, KV, S, D), 7.0, device="cuda", dtype=dt)
    vc = torch.full((B + 1, KV, S, D), 7.0, device="cuda", dtype=dt)
    p = torch.tensor([pos], device="cuda") if device_pos else pos
    q = qk_norm_rope_cache(qkv, qn, kn, cos, sin, num_heads=H, num_kv_heads=KV, head_dim=D, k_cache=kc,
                           v_cache=vc, pos=p)
    # the engine's eager lines
    qf, kf, vf = qkv.split([H * D, KV * D, KV * D], dim=-1)
    eq = qn(qf.view(B, 1, H, D)).transpose(1, 2)
    ek = kn(kf.view(B, 1, KV, D)).transpose(1, 2)
    eq, ek = rope(eq, cos[pos:pos + 1], sin[pos:pos + 1]), rope(ek, cos[pos:pos + 1], sin[pos:pos + 1])
    ev = vf.view(B, 1, KV, D).transpose(1, 2)
    assert q.shape == (B, H, 1, D)
    _ulp_close(q, eq, dt)
    _ulp_close(kc[:B, :, pos:pos + 1], ek, dt)
    assert torch.equal(vc[:B, :, pos:pos + 1], ev)
    untouched = torch.ones_like(kc, dtype=torch.bool)
    untouched[:B, :, pos] = False
    assert (kc[untouched] == 7).all() and (vc[untouched] == 7).all()


def test_glue_rejects_bad_calls():
    from llms_b200 import _capi
    lib = _capi.lib
    x = torch.zeros(2, 100, device="cuda", dtype=torch.bfloat16)  # 200-byte rows: not 16-byte aligned
    w = torch.ones(100, device="cuda", dtype=torch.bfloat16)
    st = lib.b200mm_rmsnorm(x.data_ptr(), 100, None, 0, None, 0, w.data_ptr(), x.data_ptr(), 100, 2, 100,
                            1e-6, 2, None)
    assert st != 0
    st = lib.b200mm_qk_norm_rope(x.data_ptr(), 100, 1, 3, 2, 96, w.data_ptr(), w.data_ptr(), w.data_ptr(),
                                 w.data_ptr(), 4, 0, None, x.data_ptr(), 0, 96, x.data_ptr(), 0, 0, 96,
                                 x.data_ptr(), 0, 0, 96, 1e-6, 2, None)
    assert st == 1  # D = 96 and H % KV != 0: shape refused before any launch
