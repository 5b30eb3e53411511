"""Generate golden outputs by running the REFERENCE engine's own modules.

Run in a container where the reference checkout exists:

    LLMS_REF=/path/to/aaholmes-llms python tests/golden/make_golden.py

Inputs come from ``oracle/inputs.py`` (seeded numpy), so the fixtures hold
only the reference's OUTPUTS (plus the few values the reference module itself
produced inside its forward, e.g. the normalised q of an MLA step).  Every
forward runs in float32 on CPU on bf16-representable inputs, i.e. the
"fp32-accumulated reference on identical inputs" the parity tests compare
against.  Values are captured with forward hooks on the reference modules:
  * gate-up-SiLU: the input of ``FFN.down`` inside ``FFN.forward``
    (engine/model.py:36-37);
  * QKV: the outputs of ``Attention.q/k/v`` inside ``Attention.forward``
    (engine/attention.py:119-121);
  * MLA decode: the output of ``q_norm`` and the input of ``o`` inside
    ``MLAttention.forward`` (engine/mla.py:195-265), T == 1;
  * ``down``: the input and output of ``FFN.down`` inside ``FFN.forward``
    (engine/model.py:37);
  * Qwen3-8B int8 decode step: the logits and ``greedy`` argmax
    (engine/sampler.py:17-19) of the reference ``Qwen3Model``
    (engine/model.py:76-150), built from a synthetic ``PretrainedConfig``
    (pattern tests/_tiny.py:35-49) at the 8B widths with 2 layers and a
    4096-row vocabulary, its int8 projections dequantised (W = q * s), after a
    prefill; the weights are ``oracle.inputs.cfg5_model`` (regenerated, not
    stored);
  * MLA module steps: the outputs of the reference ``MLAttention``
    (engine/mla.py:173-265) at the Qwen3-4B MLA point over a 20-token prefill
    and three decode steps on the same cache (weights and inputs from
    ``oracle.inputs.mla_module`` / ``mla_steps``);
  * GQA decode: the input and output of ``o`` of ``Attention.forward`` on its default
    single-query path (repeat_interleave + SDPA, engine/attention.py:147-150),
    and the q / K / V that path sees, captured through the module's own decode
    seam (``decode_attn_op``, :138-145) in a second, identical forward.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
if "LLMS_REF" not in os.environ:
    sys.exit("set LLMS_REF to the reference checkout (the directory holding src/engine)")
REF = Path(os.environ["LLMS_REF"])
sys.path.insert(0, str(REF / "src"))

from engine.attention import Attention, RMSNorm, build_rope_tables  # noqa: E402
from engine.kv_cache import KVCache  # noqa: E402
from engine.mla import MLAKVCache, MLAttention  # noqa: E402
from engine.model import FFN, Qwen3Model  # noqa: E402
from engine.sampler import greedy  # noqa: E402

from oracle import inputs as I  # noqa: E402


def capture_input(module):
    box = {}
    h = module.register_forward_hook(lambda m, args, out: box.__setitem__("v", args[0].detach().clone()))
    return box, h


def capture_output(module):
    box = {}
    h = module.register_forward_hook(lambda m, args, out: box.__setitem__("v", out.detach().clone()))
    return box, h


def ref_gate_up(x, wg, wu):
    N, K = wg.shape
    ffn = FFN(K, N)
    with torch.no_grad():
        ffn.gate.weight.copy_(torch.from_numpy(wg))
        ffn.up.weight.copy_(torch.from_numpy(wu))
    box, h = capture_input(ffn.down)
    with torch.no_grad():
        ffn(torch.from_numpy(x))
    h.remove()
    return box["v"].numpy()


def ref_down(x, seed=12, hidden=256, inter=768):
    """The reference FFN (engine/model.py:27-37) on x [M, hidden]: the input
    and output of its ``down`` projection, and the down weight."""
    torch.manual_seed(seed)
    ffn = FFN(hidden, inter)
    bi, h1 = capture_input(ffn.down)
    bo, h2 = capture_output(ffn.down)
    with torch.no_grad():
        ffn(torch.from_numpy(x))
    h1.remove()
    h2.remove()
    return dict(h=bi["v"].numpy(), w=ffn.down.weight.detach().numpy().copy(), y=bo["v"].numpy())


def ref_qkv(x, w, n_q, n_k, head_dim=128):
    K = w.shape[1]
    attn = Attention(hidden_size=K, num_heads=n_q // head_dim, num_kv_heads=n_k // head_dim,
                     head_dim=head_dim, rms_eps=1e-6)
    with torch.no_grad():
        attn.q.weight.copy_(torch.from_numpy(w[:n_q]))
        attn.k.weight.copy_(torch.from_numpy(w[n_q:n_q + n_k]))
        attn.v.weight.copy_(torch.from_numpy(w[n_q + n_k:]))
    bq, h1 = capture_output(attn.q)
    bk, h2 = capture_output(attn.k)
    bv, h3 = capture_output(attn.v)
    M = x.shape[0]
    cache = KVCache.alloc(num_layers=1, max_batch=1, num_kv_heads=n_k // head_dim, max_seq_len=M,
                          head_dim=head_dim, dtype=torch.float32, device="cpu")
    cos = torch.ones(M, head_dim)
    sin = torch.zeros(M, head_dim)
    with torch.no_grad():
        attn(torch.from_numpy(x)[None], kv_cache=cache, layer_idx=0, cos=cos, sin=sin, start_pos=0)
    for h in (h1, h2, h3):
        h.remove()
    return bq["v"][0].numpy(), bk["v"][0].numpy(), bv["v"][0].numpy()


def ref_mla_decode(d, L, *, H, KV, D, DR, R, theta, eps, seed, knorm_noise):
    """Run MLAttention.forward for one token at position L-1 on a cache whose
    rows 0..L-2 are the seeded inputs.  Returns (q_normed, new c row, new kr
    row, attention output before o, rope tables for positions 0..L-1)."""
    B = d["q"].shape[0]
    hidden = 64
    torch.manual_seed(seed)
    mla = MLAttention(hidden_size=hidden, num_heads=H, num_kv_heads=KV, head_dim=D, rms_eps=eps, rank=R,
                      d_rope=DR, max_position_embeddings=L + 1, rope_theta=theta, qk_norm_mode="single")
    with torch.no_grad():
        for lin in (mla.q, mla.dkv, mla.kr, mla.o):
            if lin is not None:
                lin.weight.copy_(torch.randn_like(lin.weight) * 0.1)
        if mla.uk_nope is not None:
            mla.uk_nope.weight.copy_(torch.from_numpy(d["w_uk"].reshape(KV * (D - DR), R)))
        mla.uv.weight.copy_(torch.from_numpy(d["w_uv"].reshape(KV * D, R)))
        kw = torch.from_numpy(d["k_norm_w"]).clone()
        if knorm_noise:
            kw = kw + knorm_noise * torch.randn(D)
        mla.k_norm.weight.copy_(kw)
    cache = MLAKVCache.alloc(num_layers=1, max_batch=B, num_kv_heads=KV, max_seq_len=L + 1, rank=R,
                             d_rope=DR, dtype=torch.float32, device="cpu")
    cache.c_kv[0][:, : L - 1] = torch.from_numpy(d["c_kv"][:, : L - 1])
    if DR > 0:
        cache.k_rope_pre[0][:, : L - 1] = torch.from_numpy(d["k_rope_pre"][:, : L - 1])
    bq, h1 = capture_output(mla.q_norm)
    bo, h2 = capture_input(mla.o)
    x = torch.randn(B, 1, hidden)
    with torch.no_grad():
        mla(x, kv_cache=cache, layer_idx=0, start_pos=L - 1)
    h1.remove()
    h2.remove()
    out = dict(
        q=bq["v"][:, 0].numpy(),
        c_new=cache.c_kv[0][:, L - 1].numpy().copy(),
        attn=bo["v"][:, 0].reshape(B, H, D).numpy(),
        k_norm_w=mla.k_norm.weight.detach().numpy().copy(),
    )
    if DR > 0:
        out["kr_new"] = cache.k_rope_pre[0][:, L - 1].numpy().copy()
        out["rope_cos"] = mla.rope_cos[:L].numpy().copy()
        out["rope_sin"] = mla.rope_sin[:L].numpy().copy()
    return out


def ref_gqa_decode(*, B, H, KV, D, n_prefill, seed, hidden=64):
    """One decode step (T == 1) of the reference ``Attention`` after a prefill
    of ``n_prefill`` tokens; returns q [B, H, D], K / V [B, KV, L, D] (L =
    n_prefill + 1, the whole cache), the softmax scale and the attention
    output [B, H, D] of the default path."""
    torch.manual_seed(seed)
    attn = Attention(hidden_size=hidden, num_heads=H, num_kv_heads=KV, head_dim=D, rms_eps=1e-6)
    L = n_prefill + 1
    cache = KVCache.alloc(num_layers=1, max_batch=B, num_kv_heads=KV, max_seq_len=L, head_dim=D,
                          dtype=torch.float32, device="cpu")
    cos, sin = build_rope_tables(D, L, base=1e6, dtype=torch.float32)
    x0 = torch.randn(B, n_prefill, hidden)
    x1 = torch.randn(B, 1, hidden)
    with torch.no_grad():
        attn(x0, kv_cache=cache, layer_idx=0, cos=cos[:n_prefill], sin=sin[:n_prefill], start_pos=0)
        box, h = capture_input(attn.o)
        bo, h2 = capture_output(attn.o)
        attn(x1, kv_cache=cache, layer_idx=0, cos=cos[n_prefill:L], sin=sin[n_prefill:L], start_pos=n_prefill)
        h.remove()
        h2.remove()
        grab = {}

        def spy(q, full_k, full_v, *, scale, layer_idx):
            grab.update(q=q.clone(), k=full_k.clone(), v=full_v.clone(), scale=scale)
            return torch.zeros_like(q)

        attn.decode_attn_op = spy
        attn(x1, kv_cache=cache, layer_idx=0, cos=cos[n_prefill:L], sin=sin[n_prefill:L], start_pos=n_prefill)
    return dict(q=grab["q"][:, :, 0].numpy().copy(), k=grab["k"].numpy().copy(), v=grab["v"].numpy().copy(),
                scale=np.array([grab["scale"]], np.float32),
                out=box["v"].view(B, H, D).numpy().copy(),
                o_w=attn.o.weight.detach().numpy().copy(), o_y=bo["v"].numpy().copy())


def ref_qwen3_int8_step(*, layers=2, vocab=4096, batch=16, prompt=6):
    """The reference engine's decode step on the dequantised config-5 model:
    prefill ``prompt`` tokens, then one new token per row; returns the decode
    step's logits [batch, vocab], their greedy argmax and the prefill's last
    logits."""
    from transformers import PretrainedConfig

    cfg = PretrainedConfig(vocab_size=vocab, hidden_size=4096, num_hidden_layers=layers, num_attention_heads=32,
                           num_key_value_heads=8, head_dim=128, intermediate_size=12288,
                           max_position_embeddings=64, rms_norm_eps=1e-6, tie_word_embeddings=False,
                           rope_theta=1e6, attention_bias=False)
    st = I.cfg5_model(layers=layers, vocab=vocab)
    deq = lambda q, s: torch.from_numpy(q.astype(np.float32) * st[s][:, None])
    sd = {"embed.weight": torch.from_numpy(st["embed.weight"]),
          "lm_head.weight": torch.from_numpy(st["lm_head.weight"]),
          "final_norm.weight": torch.ones(4096)}
    for i in range(layers):
        p = f"layers.{i}."
        w = deq(st[p + "attn.q_qkv"], p + "attn.s_qkv")
        sd[p + "attn.q.weight"], sd[p + "attn.k.weight"], sd[p + "attn.v.weight"] = w.split([4096, 1024, 1024])
        sd[p + "attn.o.weight"] = torch.from_numpy(st[p + "attn.o.weight"])
        sd[p + "ffn.gate.weight"] = deq(st[p + "ffn.qg"], p + "ffn.sg")
        sd[p + "ffn.up.weight"] = deq(st[p + "ffn.qu"], p + "ffn.su")
        sd[p + "ffn.down.weight"] = torch.from_numpy(st[p + "ffn.down.weight"])
        for n in ("norm1.weight", "norm2.weight"):
            sd[p + n] = torch.ones(4096)
        for n in ("attn.q_norm.weight", "attn.k_norm.weight"):
            sd[p + n] = torch.ones(128)
    model = Qwen3Model(cfg)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rope" in k for k in missing), (missing, unexpected)
    model.eval()
    ids, nxt = I.cfg5_tokens(batch, prompt, vocab)
    cache = model.alloc_cache(prompt + 2, max_batch=batch, dtype=torch.float32, device="cpu")
    with torch.no_grad():
        pre = model(torch.from_numpy(ids), cache, start_pos=0)[:, -1]
        logits = model(torch.from_numpy(nxt), cache, start_pos=prompt)[:, -1]
    return dict(logits=logits.numpy().copy(), argmax=greedy(logits).numpy().astype(np.float32),
                prefill_logits=pre.numpy().copy())


def ref_mla_prefill_decode(*, B=2, prefill=20, decode=3, hidden=2560):
    """The reference ``MLAttention`` (engine/mla.py:173-265) at the Qwen3-4B
    MLA point (H 32, KV 8, D 128, d_rope 32, rank 256, theta 1e6) with the
    weights of ``oracle.inputs.mla_module``: a prefill of ``prefill`` tokens,
    then ``decode`` single-token steps on the same cache.  Returns the last
    two prefill output rows and every decode step's output."""
    mla = MLAttention(hidden_size=hidden, num_heads=32, num_kv_heads=8, head_dim=128, rms_eps=1e-6, rank=256,
                      d_rope=32, max_position_embeddings=64, rope_theta=1e6, qk_norm_mode="single")
    mla.load_state_dict({k: torch.from_numpy(v) for k, v in I.mla_module(hidden).items()})
    x0, xs = I.mla_steps(B, prefill, decode, hidden)
    cache = MLAKVCache.alloc(num_layers=1, max_batch=B, num_kv_heads=8, max_seq_len=prefill + decode + 1, rank=256,
                             d_rope=32, dtype=torch.float32, device="cpu")
    with torch.no_grad():
        pre = mla(torch.from_numpy(x0), kv_cache=cache, layer_idx=0, start_pos=0)
        outs = [mla(torch.from_numpy(xs[i]), kv_cache=cache, layer_idx=0, start_pos=prefill + i)
                for i in range(decode)]
    return dict(prefill_tail=pre[:, -2:].numpy().copy(), decode=torch.stack(outs).numpy().copy())


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}

    x, wg, wu = I.cfg1()
    out["cfg1_gate_up"] = ref_gate_up(x, wg, wu)

    for M in (1, 4):
        x, w = I.cfg2(M)
        q, k, v = ref_qkv(x, w, 4096, 1024)
        out[f"cfg2_m{M}_q"], out[f"cfg2_m{M}_k"], out[f"cfg2_m{M}_v"] = q, k, v
        x, wg, wu = I.cfg3(M)
        out[f"cfg3_m{M}_gate_up"] = ref_gate_up(x, wg, wu)

    # int8 weight-only: dequantise, then the reference modules
    for M in (1, 4):
        lay = I.cfg5_layer(M=M)
        wq = lay["qkv_q"].astype(np.float32) * lay["qkv_s"][:, None]
        q, k, v = ref_qkv(lay["x"], wq, 4096, 1024)
        out[f"cfg5_m{M}_qkv"] = np.concatenate([q, k, v], axis=-1)
        wg = lay["gate_q"].astype(np.float32) * lay["gate_s"][:, None]
        wu = lay["up_q"].astype(np.float32) * lay["up_s"][:, None]
        out[f"cfg5_m{M}_gate_up"] = ref_gate_up(lay["x"], wg, wu)

    mla_cases = {
        # name: (B, L, dims, knorm noise)
        "mla_4b_b2_l37": (2, 37, dict(H=32, KV=8, D=128, DR=32, R=256), 0.0),
        "mla_4b_b1_l300_knorm": (1, 300, dict(H=32, KV=8, D=128, DR=32, R=256), 0.1),
        "mla_tiny_dr8": (3, 9, dict(H=4, KV=2, D=16, DR=8, R=12), 0.1),
        "mla_tiny_dr0": (2, 5, dict(H=4, KV=2, D=16, DR=0, R=12), 0.1),
        "mla_tiny_drfull": (2, 6, dict(H=4, KV=2, D=16, DR=16, R=12), 0.1),
    }
    for name, (B, L, dims, noise) in mla_cases.items():
        d = I.cfg4(B, L, **dims)
        r = ref_mla_decode(d, L, theta=1e6, eps=1e-6, seed=5, knorm_noise=noise, **dims)
        for k_, v_ in r.items():
            out[f"{name}__{k_}"] = v_

    # the bias-free projections behind o / down (engine/attention.py:163,
    # engine/model.py:37): the reference FFN's own down input and output
    rng = np.random.default_rng(12)
    for k_, v_ in ref_down(rng.standard_normal((3, 256), dtype=np.float32)).items():
        out[f"down_m3__{k_}"] = v_

    gqa_cases = {
        # name: (B, H, KV, D, prefill tokens)
        "gqa_b2_h8_kv2_d128_l38": (2, 8, 2, 128, 37),
        "gqa_b3_h12_kv4_d64_l70": (3, 12, 4, 64, 69),
        "gqa_b1_h4_kv4_d32_l5": (1, 4, 4, 32, 4),
    }
    for name, (B, H, KV, D, n) in gqa_cases.items():
        for k_, v_ in ref_gqa_decode(B=B, H=H, KV=KV, D=D, n_prefill=n, seed=11).items():
            out[f"{name}__{k_}"] = v_

    for k_, v_ in ref_mla_prefill_decode().items():
        out[f"mla_4b_module_steps__{k_}"] = v_

    for k_, v_ in ref_qwen3_int8_step().items():
        out[f"qwen3_8b_int8_l2__{k_}"] = v_

    np.savez_compressed(HERE / "golden.npz", **{k: np.asarray(v, np.float32) for k, v in out.items()})
    print(f"wrote {HERE / 'golden.npz'} with {len(out)} arrays")


if __name__ == "__main__":
    main()
