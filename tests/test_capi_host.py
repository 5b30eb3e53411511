"""C ABI checks that need no GPU: the library loads, exports every symbol
the header declares, and rejects invalid calls before touching a device."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "b200mm.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200mm_\w+)\s*\(", text)))


def test_library_exports_header_symbols():
    from llms_b200 import _capi
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(_capi.lib, s), f"{s} declared in include/b200mm.h but not exported"
        assert s in _capi.SIGNATURES, f"{s} has no ctypes signature"


def test_status_strings_and_version():
    from llms_b200 import _capi
    assert _capi.lib.b200mm_abi_version() == 2
    assert _capi.lib.b200mm_status_string(0) == b"ok"
    for code in range(1, 9):
        assert _capi.lib.b200mm_status_string(code) not in (b"ok", b"unknown status")
    assert _capi.lib.b200mm_status_string(99) == b"unknown status"


def test_null_pointers_and_bad_shapes_rejected_before_launch():
    from llms_b200 import _capi
    L = _capi.lib
    before = L.b200mm_launch_count()
    assert L.b200mm_gate_up_silu(None, 64, None, 64, None, 64, None, 64, 1, 64, 64, 2, None) == 5
    fake = ctypes.c_void_p(16)
    # K < 1, N < 1, ld < K, bad dtype
    assert L.b200mm_qkv(fake, 64, fake, 64, fake, 96, 1, 96, 0, 2, None) == 1
    assert L.b200mm_qkv(fake, 64, fake, 64, fake, 96, 1, 0, 64, 2, None) == 1
    assert L.b200mm_qkv(fake, 32, fake, 64, fake, 96, 1, 96, 64, 2, None) == 1
    assert L.b200mm_qkv(fake, 64, fake, 64, fake, 96, 1, 96, 64, 7, None) == 3
    # int8 with fp32 activations is not a supported combination
    assert L.b200mm_qkv_w8(fake, 64, fake, fake, 64, fake, 96, 1, 96, 64, 0, None) == 3
    # M == 0 is a successful no-op
    assert L.b200mm_qkv(fake, 64, fake, 64, fake, 96, 0, 96, 64, 2, None) == 0
    shp = _capi.MlaShape(B=1, H=32, KV=8, D=128, DR=33, R=256, dtype=2, eps=1e-6)  # odd d_rope
    assert L.b200mm_mla_decode_workspace_size(ctypes.byref(shp), 10) == 0
    shp.DR = 32
    assert L.b200mm_mla_decode_workspace_size(ctypes.byref(shp), 10) > 0
    assert L.b200mm_launch_count() == before


def test_shim_rejects_with_reference_messages():
    """Same ValueError messages as reference tests/test_kernels_fused_ffn.py:209-229
    and tests/test_kernels_fused_qkv.py:253-277 (host-side validation, CPU tensors)."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    x = torch.randn(2, 64)
    Wg = torch.randn(128, 64)
    with pytest.raises(ValueError, match="Wg shape.*Wu shape"):
        triton_fused_gate_up_silu(x, Wg, torch.randn(127, 64))
    with pytest.raises(ValueError, match="Wg shape.*Wu shape"):
        triton_fused_gate_up_silu(x, Wg, torch.randn(128, 63))
    W3 = torch.randn(2, 128, 64)
    with pytest.raises(ValueError, match="Wg must be 2D"):
        triton_fused_gate_up_silu(x, W3, W3)
    with pytest.raises(ValueError, match="x last dim.*Wg.shape"):
        triton_fused_gate_up_silu(torch.randn(2, 63), Wg, Wg)

    W_qkv = torch.randn(96, 64)
    with pytest.raises(ValueError, match="n_q .* 2.n_k"):
        triton_fused_qkv(x, W_qkv, n_q=64, n_k=15)
    with pytest.raises(ValueError, match="x last dim .* W_qkv"):
        triton_fused_qkv(torch.randn(2, 63), W_qkv, n_q=64, n_k=16)
    with pytest.raises(ValueError, match="W_qkv must be 2D"):
        triton_fused_qkv(x, torch.randn(2, 96, 64), n_q=64, n_k=16)


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: a valid call on CPU tensors raises instead of computing."""
    from llms_b200.kernels import triton_fused_gate_up_silu, triton_fused_qkv
    x = torch.randn(2, 64)
    W = torch.randn(96, 64)
    with pytest.raises(RuntimeError, match="no CPU path"):
        triton_fused_gate_up_silu(x, W, W)
    with pytest.raises(RuntimeError, match="no CPU path"):
        triton_fused_qkv(x, W, n_q=64, n_k=16)


def test_linear_and_gqa_entry_points_validate_before_launch():
    """b200mm_linear(_w8) and b200mm_gqa_decode reject invalid calls with the
    documented status codes before touching a device (no GPU here: a valid
    call reaches the device check and returns B200MM_ERR_DEVICE)."""
    from llms_b200 import _capi
    L = _capi.lib
    before = L.b200mm_launch_count()
    fake = ctypes.c_void_p(256)
    OK, SHAPE, DTYPE, ARG, WS, DEV = 0, 1, 3, 5, 6, 7
    # plain projection: same checks as the QKV entry point
    assert L.b200mm_linear(None, 64, fake, 64, fake, 32, 1, 32, 64, 2, None) == ARG
    assert L.b200mm_linear(fake, 64, fake, 64, fake, 32, 1, 32, 0, 2, None) == SHAPE
    assert L.b200mm_linear(fake, 64, fake, 64, fake, 32, 1, 32, 64, 9, None) == DTYPE
    assert L.b200mm_linear(fake, 64, fake, 64, fake, 32, 0, 32, 64, 2, None) == OK
    assert L.b200mm_linear_w8(fake, 64, fake, None, 64, fake, 32, 1, 32, 64, 2, None) == ARG
    # GQA decode: workspace size, then argument checks in order
    ws = L.b200mm_gqa_decode_workspace_size(2, 32, 8, 128, 1000)
    assert ws > 0 and ws % 256 == 0
    assert L.b200mm_gqa_decode_workspace_size(2, 32, 7, 128, 1000) == 0   # H % KV != 0
    assert L.b200mm_gqa_decode_workspace_size(2, 32, 8, 128, 0) == 0      # no tokens
    assert L.b200mm_gqa_decode_workspace_size(2, 32, 8, 127, 10) == 0     # odd head dim
    good = dict(q_sb=32 * 128, q_sh=128, k_sb=8 * 1024 * 128, k_sh=1024 * 128, k_st=128)

    def call(q=fake, k=fake, v=fake, out=fake, B=2, H=32, KV=8, D=128, Lc=1000, scale=0.088, dtype=2,
             wsp=ctypes.c_void_p(4096), wsb=ws, k_st=128):
        return L.b200mm_gqa_decode(q, good["q_sb"], good["q_sh"], k, good["k_sb"], good["k_sh"], k_st,
                                   v, good["k_sb"], good["k_sh"], k_st, out, good["q_sb"], good["q_sh"],
                                   B, H, KV, D, Lc, scale, dtype, wsp, wsb, None)

    assert call(dtype=5) == DTYPE
    assert call(KV=7) == SHAPE
    assert call(q=None) == ARG
    assert call(scale=0.0) == ARG
    assert call(k_st=64) == SHAPE                    # token stride shorter than a row
    assert call(B=0) == OK                           # empty batch: no-op
    assert call(wsb=ws - 1) == WS                    # workspace too small
    assert call(wsp=ctypes.c_void_p(4096 + 16)) == WS  # workspace not 256-byte aligned
    assert call() == DEV                             # valid: stops at the device check here
    assert L.b200mm_launch_count() == before


def test_new_ops_check_arguments_on_the_host():
    """b200_linear / int8_linear / b200_decode_attn validate shapes and dtypes
    before any device work, and refuse CPU tensors (no CPU path)."""
    from llms_b200.kernels import b200_decode_attn, b200_linear, int8_linear
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="W must be 2D"):
        b200_linear(x, torch.zeros(64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="x last dim"):
        b200_linear(x, torch.zeros(8, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="share a dtype"):
        b200_linear(x, torch.zeros(8, 64, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="no CPU path"):
        b200_linear(x, torch.zeros(8, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="int8"):
        int8_linear(x, torch.zeros(8, 64, dtype=torch.bfloat16), torch.ones(8))
    with pytest.raises(ValueError, match="float32 of shape"):
        int8_linear(x, torch.zeros(8, 64, dtype=torch.int8), torch.ones(7))
    q = torch.zeros(2, 8, 1, 64, dtype=torch.bfloat16)
    k = torch.zeros(2, 2, 10, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=r"\(B, H, 1, D\)"):
        b200_decode_attn(q[:, :, 0], k, k, scale=0.1)
    with pytest.raises(ValueError, match="does not match"):
        b200_decode_attn(q, torch.zeros(2, 3, 10, 64, dtype=torch.bfloat16),
                         torch.zeros(2, 3, 10, 64, dtype=torch.bfloat16), scale=0.1)
    with pytest.raises(RuntimeError, match="no CPU path"):
        b200_decode_attn(q, k, k, scale=0.1)


def test_peer_out_mirror_matches_header_layout():
    """llms_b200._capi.PeerOut has b200mm_peer_out's layout (the C side checks
    the same offsets in tests/c/abi_check.c)."""
    import ctypes
    from llms_b200._capi import PeerOut
    assert ctypes.sizeof(PeerOut) == 200
    assert PeerOut.ld_dst.offset == 64 and PeerOut.nparts.offset == 96
    assert PeerOut.flags.offset == 112 and PeerOut.err.offset == 192
