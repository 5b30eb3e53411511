"""Pin the CPU oracle against golden outputs of the reference engine's own
modules (tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest

from oracle import inputs as I
from oracle import reference_math as O


def _close(a, e, rtol, atol):
    np.testing.assert_allclose(np.asarray(a, np.float64), np.asarray(e, np.float64), rtol=rtol, atol=atol)


def test_cfg1_gate_up(golden):
    x, wg, wu = I.cfg1()
    _close(O.gate_up_silu(x, wg, wu), golden["cfg1_gate_up"], 1e-4, 1e-6)


@pytest.mark.parametrize("M", [1, 4])
def test_cfg2_qkv(golden, M):
    x, w = I.cfg2(M)
    q, k, v = O.qkv(x, w, 4096, 1024)
    for name, got in (("q", q), ("k", k), ("v", v)):
        _close(got, golden[f"cfg2_m{M}_{name}"], 1e-4, 1e-5)


@pytest.mark.parametrize("M", [1, 4])
def test_cfg3_gate_up(golden, M):
    x, wg, wu = I.cfg3(M)
    _close(O.gate_up_silu(x, wg, wu), golden[f"cfg3_m{M}_gate_up"], 1e-4, 1e-5)


@pytest.mark.parametrize("M", [1, 4])
def test_cfg5_int8(golden, M):
    lay = I.cfg5_layer(M=M)
    q, k, v = O.qkv(lay["x"], O.dequant(lay["qkv_q"], lay["qkv_s"]), 4096, 1024)
    _close(np.concatenate([q, k, v], -1), golden[f"cfg5_m{M}_qkv"], 1e-4, 1e-5)
    g = O.gate_up_silu(lay["x"], O.dequant(lay["gate_q"], lay["gate_s"]), O.dequant(lay["up_q"], lay["up_s"]))
    _close(g, golden[f"cfg5_m{M}_gate_up"], 1e-4, 5e-5)


MLA_CASES = {
    "mla_4b_b2_l37": (2, 37, dict(H=32, KV=8, D=128, DR=32, R=256)),
    "mla_4b_b1_l300_knorm": (1, 300, dict(H=32, KV=8, D=128, DR=32, R=256)),
    "mla_tiny_dr8": (3, 9, dict(H=4, KV=2, D=16, DR=8, R=12)),
    "mla_tiny_dr0": (2, 5, dict(H=4, KV=2, D=16, DR=0, R=12)),
    "mla_tiny_drfull": (2, 6, dict(H=4, KV=2, D=16, DR=16, R=12)),
}


def mla_case(golden, name):
    """Inputs of a golden MLA case: seeded cache rows 0..L-2 plus the new
    token's row L-1 and the normalised q captured from the reference module."""
    B, L, dims = MLA_CASES[name]
    d = I.cfg4(B, L, **dims)
    d["c_kv"][:, L - 1] = golden[f"{name}__c_new"]
    if dims["DR"] > 0:
        d["k_rope_pre"][:, L - 1] = golden[f"{name}__kr_new"]
    d["q"] = golden[f"{name}__q"]
    d["k_norm_w"] = golden[f"{name}__k_norm_w"]
    return B, L, dims, d


@pytest.mark.parametrize("name", list(MLA_CASES))
def test_mla_decode(golden, name):
    B, L, dims, d = mla_case(golden, name)
    inv = O.mla_inv_freq(dims["D"], dims["DR"], 1e6)
    out = O.mla_decode(d["q"], d["c_kv"], d["k_rope_pre"], d["w_uk"], d["w_uv"], d["k_norm_w"], 1e-6, inv, L)
    _close(out, golden[f"{name}__attn"], 2e-4, 2e-5)


@pytest.mark.parametrize("name", ["mla_4b_b2_l37", "mla_tiny_dr8"])
def test_mla_rope_tables(golden, name):
    """The reference's partial-RoPE table (engine/mla.py:151-171, theta=1e6,
    head_dim 128, d_rope 32 for the 4B case) matches the oracle's."""
    B, L, dims = MLA_CASES[name]
    cos, sin = O.rope_cos_sin(np.arange(L), O.mla_inv_freq(dims["D"], dims["DR"], 1e6))
    _close(cos, golden[f"{name}__rope_cos"], 0, 2e-6)
    _close(sin, golden[f"{name}__rope_sin"], 0, 2e-6)


@pytest.mark.parametrize("name", ["gqa_b2_h8_kv2_d128_l38", "gqa_b3_h12_kv4_d64_l70", "gqa_b1_h4_kv4_d32_l5"])
def test_gqa_decode(golden, name):
    """The GQA decode oracle vs the reference Attention's default single-query
    path, on the q / K / V that path saw."""
    g = lambda k: golden[f"{name}__{k}"]
    _close(O.gqa_decode(g("q"), g("k"), g("v"), float(g("scale")[0])), g("out"), 1e-5, 1e-6)


def test_linear_down_and_o(golden):
    """The bias-free projection oracle vs the reference's own ``FFN.down``
    (engine/model.py:37) and ``Attention.o`` (engine/attention.py:163)
    inputs and outputs."""
    _close(O.linear(golden["down_m3__h"], golden["down_m3__w"]), golden["down_m3__y"], 1e-5, 1e-6)
    for name in ("gqa_b2_h8_kv2_d128_l38", "gqa_b3_h12_kv4_d64_l70", "gqa_b1_h4_kv4_d32_l5"):
        out = golden[f"{name}__out"]
        B, H, D = out.shape
        _close(O.linear(out.reshape(B, 1, H * D), golden[f"{name}__o_w"]), golden[f"{name}__o_y"], 1e-5, 1e-6)


def test_mla_module_prefill_math_vs_reference(golden):
    """B200MLAttention's restated prefill math (used when the module was not
    built by wrapping a reference MLAttention) equals the reference module's
    prefill on the same weights (CPU, fp32; the decode steps are checked on
    the GPU in tests/test_gpu_mla.py)."""
    import torch
    from llms_b200.mla import B200MLAttention

    class Cache:
        def __init__(self, B, S):
            self.c_kv = [torch.zeros(B, S, 256)]
            self.k_rope_pre = [torch.zeros(B, S, 8, 32)]

    m = B200MLAttention(hidden_size=2560, num_heads=32, num_kv_heads=8, head_dim=128, rms_eps=1e-6, rank=256,
                        d_rope=32, max_position_embeddings=64, rope_theta=1e6)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in I.mla_module().items()})
    x0, _ = I.mla_steps()
    with torch.no_grad():
        y = m._eager(torch.from_numpy(x0), kv_cache=Cache(2, 24), layer_idx=0, start_pos=0)
    _close(y[:, -2:].numpy(), golden["mla_4b_module_steps__prefill_tail"], 1e-4, 1e-5)


def test_mla_module_rejects_cpu_tensors():
    """No CPU path: the drop-in module raises on CPU inputs."""
    import torch
    from llms_b200.mla import B200MLAttention
    m = B200MLAttention(hidden_size=64, num_heads=4, num_kv_heads=2, head_dim=16, rms_eps=1e-6, rank=32,
                        d_rope=8, max_position_embeddings=16, rope_theta=1e4)
    with pytest.raises(RuntimeError, match="CPU"):
        m(torch.zeros(1, 1, 64), kv_cache=None, layer_idx=0, start_pos=0)
