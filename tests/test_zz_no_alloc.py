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


def test_noalloc_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200 import _capi, mla

    lib = _capi.lib
    H, KV, D, DR, R = 32, 8, 128, 32, 256
    for B, L, seed in ((4, 1000, 11), (2, 3000, 12)):
        d = I.cfg4(B, L, seed=seed)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
        c, kr, wuk, wuv, q = to(d["c_kv"]), to(d["k_rope_pre"]), to(d["w_uk"]), to(d["w_uv"]), to(d["q"])
        kw = torch.ones(D, device="cuda")
        inv = mla.rope_inv_freq(D, DR, 1e6, "cuda")
        ks, kz = mla.mla_sidebands(c, kr, wuk, kw, inv, B=B, L=L, num_kv_heads=KV, head_dim=D, eps=1e-6)
        shp = _capi.MlaShape(B=B, H=H, KV=KV, D=D, DR=DR, R=R, dtype=2, eps=1e-6)
        stream = torch.cuda.current_stream().cuda_stream

        ref = torch.empty(B, H, D, device="cuda", dtype=torch.bfloat16)
        nbytes = lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L)
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
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_b200 import _capi

    lib = _capi.lib
    B, L = 256, 32768  # needs far more than the library's 8 MiB array
    shp = _capi.MlaShape(B=B, H=32, KV=8, D=128, DR=32, R=256, dtype=2, eps=1e-6)
    assert lib.b200mm_mla_decode_workspace_size(ctypes.byref(shp), L) > 8 << 20
    fake = ctypes.c_void_p(256)
    before = lib.b200mm_launch_count()
    st = lib.b200mm_mla_decode_noalloc(ctypes.byref(shp), fake, 4096, fake, 256 * L, 256, fake, 256 * L, 256,
                                       fake, 8 * L, 8, fake, fake, fake, fake, ctypes.c_float(0.088), L, fake,
                                       4096, None)
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
