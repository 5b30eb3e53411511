"""The allocation-free MLA decode entry point (b200mm_mla_decode_noalloc).

Some callers of this library cannot allocate device memory when they decode
(a server that hands out memory only from an arena it reserved at start-up, a
replayed CUDA graph, a plugin whose host framework owns all allocations).  The
no-alloc entry point serves them from a fixed array inside the library.  This
test checks, through the C ABI, that it returns the same output as
b200mm_mla_decode with a caller-provided workspace, on two calls in a row (the
second call reuses the array the first one left behind), and that a shape whose
workspace exceeds the array is refused without a launch.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import inputs as I
from tests.conftest import bf16_check

pytestmark = pytest.mark.gpu


def _args(shp, q, c, kz, ks, wuk, wuv, kw, inv, L, out):
    return (ctypes.byref(shp), q.data_ptr(), q.stride(0), c.data_ptr(), c.stride(0), c.stride(1),
            kz.data_ptr(), kz.stride(0), kz.stride(1), ks.data_ptr(), ks.stride(0), ks.stride(1),
            wuk.data_ptr(), wuv.data_ptr(), kw.data_ptr(), inv.data_ptr(), ctypes.c_float(128 ** -0.5), L,
            out.data_ptr(), out.stride(0))


def _case(B, L, seed):
    """Inputs on the device: the seeded oracle generator for small cases, a
    device generator for the largest (same distributions, config 4)."""
    if B * L <= 8192:
        d = I.cfg4(B, L, seed=seed)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
        return to(d["c_kv"]), to(d["k_rope_pre"]), to(d["w_uk"]), to(d["w_uv"]), to(d["q"])
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s, std=1.0: (torch.randn(*s, device="cuda", generator=g) * std).to(torch.bfloat16)
    return r(B, L, 256), r(B, L, 8, 32), r(8, 96, 256, std=0.25), r(8, 128, 256, std=0.25), r(B, 32, 128)


@pytest.mark.parametrize("B,L,seed", [(4, 1000, 11), (2, 3000, 12), (32, 32768, 13)])
def test_noalloc_matches_workspace_entry_point(B, L, seed):
    """Same output as b200mm_mla_decode with a caller workspace, on two calls
    in a row; (32, 32768) is the largest documented case and reaches the end
    of the array."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200 import _capi, mla

    lib = _capi.lib
    H, KV, D, DR, R = 32, 8, 128, 32, 256
    c, kr, wuk, wuv, q = _case(B, L, seed)
    kw = torch.ones(D, device="cuda")
    inv = mla.rope_inv_freq(D, DR, 1e6, "cuda")
    ks, kz = mla.mla_sidebands(c, kr, wuk, kw, inv, B=B, L=L, num_kv_heads=KV, head_dim=D, eps=1e-6)
    del kr
    shp = _capi.MlaShape(B=B, H=H, KV=KV, D=D, DR=DR, R=R, dtype=2, eps=1e-6)
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty(B, H, D, device="cuda", dtype=torch.bfloat16)
    nbytes = lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L)
    assert nbytes <= 8 << 20
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    st = lib.b200mm_mla_decode(*_args(shp, q, c, kz, ks, wuk, wuv, kw, inv, L, ref), ws.data_ptr(), nbytes,
                               stream)
    assert st == 0, lib.b200mm_status_string(st)

    for _ in range(2):  # two calls in a row share the library's array
        out = torch.full((B, H, D), float("nan"), device="cuda", dtype=torch.bfloat16)
        st = lib.b200mm_mla_decode_noalloc(*_args(shp, q, c, kz, ks, wuk, wuv, kw, inv, L, out), stream)
        assert st == 0, lib.b200mm_status_string(st)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        bf16_check(out.float().cpu().numpy(), ref.float().cpu().numpy().astype(np.float64))


def test_noalloc_refuses_oversized_workspace():
    """A batch whose workspace exceeds the array is refused before any launch.
    The buffers are real device tensors of the claimed shape, so nothing here
    hands the library an address it does not own."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200 import _capi, mla

    lib = _capi.lib
    B, L = 128, 64  # 128 rows of partials and absorbed queries: ~16 MiB of workspace
    shp = _capi.MlaShape(B=B, H=32, KV=8, D=128, DR=32, R=256, dtype=2, eps=1e-6)
    assert lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L) > 8 << 20
    bf = dict(device="cuda", dtype=torch.bfloat16)
    c, kz = torch.zeros(B, L, 256, **bf), torch.zeros(B, L, 8, 32, **bf)
    ks = torch.ones(B, L, 8, device="cuda")
    wuk, wuv, q = torch.zeros(8, 96, 256, **bf), torch.zeros(8, 128, 256, **bf), torch.zeros(B, 32, 128, **bf)
    kw, inv = torch.ones(128, device="cuda"), mla.rope_inv_freq(128, 32, 1e6, "cuda")
    out = torch.zeros(B, 32, 128, **bf)
    before = lib.b200mm_launch_count()
    st = lib.b200mm_mla_decode_noalloc(*_args(shp, q, c, kz, ks, wuk, wuv, kw, inv, L, out),
                                       torch.cuda.current_stream().cuda_stream)
    assert st == 6  # B200MM_ERR_WORKSPACE
    assert lib.b200mm_launch_count() == before


def test_documented_noalloc_case_fits_the_array():
    """B = 32, L = 32768 at the Qwen3-4B MLA shape is documented to fit 8 MiB."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200 import _capi

    shp = _capi.MlaShape(B=32, H=32, KV=8, D=128, DR=32, R=256, dtype=2, eps=1e-6)
    need = _capi.lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), 32768)
    assert 0 < need <= 8 << 20, need
