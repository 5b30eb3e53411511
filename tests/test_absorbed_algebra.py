"""The absorbed latent decode the CUDA kernel implements equals the
reference's reconstruct-K/V decode (float64, CPU).

score_t,h = scale * s_t,g * (qt_h . c_t + rope_{L-1}(q_r) . rope_t(w_r * kr_t,g)),
qt_h = W_uk,g^T (w_n * q_n),  out_h = W_uv,g sum_t p_t c_t.
"""

import numpy as np
import pytest

from oracle import inputs as I
from oracle import reference_math as O


def absorbed(q, c, kr, w_uk, w_uv, kw, eps, inv, L, scale):
    B, H, D = q.shape
    KV, DN, R = w_uk.shape
    DR = D - DN
    g_of = np.arange(H) // (H // KV)
    s = O.mla_kv_scales(c[:, :L], kr[:, :L] if DR else None, w_uk, eps, D)  # (B, L, KV)
    qn = kw[:DN] * q[:, :, :DN]                                   # (B, H, DN)
    qt = np.einsum("hnr,bhn->bhr", w_uk[g_of], qn)                # (B, H, R)
    sc = np.einsum("bhr,blr->bhl", qt, c[:, :L].astype(np.float64))
    if DR:
        cq, sq = O.rope_cos_sin(np.array([L - 1]), inv)
        ck, sk = O.rope_cos_sin(np.arange(L), inv)
        qr = q[..., DN:].astype(np.float64)
        qr = qr * cq[0] + O.rotate_half(qr) * sq[0]
        z = kr[:, :L].astype(np.float64) * kw[DN:]
        z = z * ck[None, :, None, :] + O.rotate_half(z) * sk[None, :, None, :]  # (B, L, KV, DR)
        sc = sc + np.einsum("bhd,blhd->bhl", qr, z[:, :, g_of])
    sc = sc * s[:, :, g_of].transpose(0, 2, 1) * scale
    p = np.exp(sc - sc.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    lat = np.einsum("bhl,blr->bhr", p, c[:, :L].astype(np.float64))
    return np.einsum("hdr,bhr->bhd", w_uv[g_of].astype(np.float64), lat)


@pytest.mark.parametrize("dims,B,L", [
    (dict(H=32, KV=8, D=128, DR=32, R=256), 2, 50),
    (dict(H=4, KV=2, D=16, DR=8, R=12), 3, 9),
    (dict(H=4, KV=2, D=16, DR=0, R=12), 2, 7),
    (dict(H=6, KV=3, D=16, DR=16, R=12), 1, 5),
])
def test_absorbed_equals_reconstruct(dims, B, L):
    d = I.cfg4(B, L, **dims)
    rng = np.random.default_rng(9)
    kw = (1 + 0.1 * rng.standard_normal(dims["D"])).astype(np.float64)
    inv = O.mla_inv_freq(dims["D"], dims["DR"], 1e6)
    ref = O.mla_decode(d["q"], d["c_kv"], d["k_rope_pre"], d["w_uk"], d["w_uv"], kw, 1e-6, inv, L)
    got = absorbed(d["q"].astype(np.float64), d["c_kv"].astype(np.float64), d["k_rope_pre"], d["w_uk"].astype(np.float64),
                   d["w_uv"], kw, 1e-6, inv, L, dims["D"] ** -0.5)
    np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-11)
