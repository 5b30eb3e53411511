"""Pin the decode harness model (``llms_b200.qwen3``) to the reference
engine: the Qwen3-8B-shaped int8 model of config 5 (2 layers, 4096-row
vocabulary), run in fp32 with dequantised weights after a prefill, gives the
logits and greedy tokens the reference ``Qwen3Model`` gave on the same
weights (tests/golden/make_golden.py, ``qwen3_8b_int8_l2__*``).  CPU only."""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import inputs as I


@pytest.fixture(scope="module")
def harness_fp32():
    from llms_b200.qwen3 import QWEN3_8B, int8_model_from_state
    shape = dataclasses.replace(QWEN3_8B, num_hidden_layers=2, vocab_size=4096, max_position_embeddings=64)
    return int8_model_from_state(I.cfg5_model(layers=2, vocab=4096), shape, device="cpu", dtype=torch.float32)


def test_harness_fp32_matches_reference_engine(golden, harness_fp32):
    from llms_b200.qwen3 import greedy
    m = harness_fp32
    ids, nxt = I.cfg5_tokens(16, 6, 4096)
    with torch.inference_mode():
        cache = m.alloc_cache(8, max_batch=16, dtype=torch.float32)
        pre = m.forward_fp32_dequant(torch.from_numpy(ids), cache, 0)[:, -1]
        logits = m.forward_fp32_dequant(torch.from_numpy(nxt), cache, 6)[:, -1]
    for got, key in ((pre, "prefill_logits"), (logits, "logits")):
        e = golden[f"qwen3_8b_int8_l2__{key}"]
        np.testing.assert_allclose(got.numpy(), e, rtol=1e-4, atol=1e-4 * np.abs(e).max())
    assert np.array_equal(greedy(logits).numpy(), golden["qwen3_8b_int8_l2__argmax"].astype(np.int64))


def test_state_loader_rejects_mismatch():
    from llms_b200.qwen3 import Qwen3Shape, int8_model_from_state
    shape = Qwen3Shape(vocab_size=64, hidden_size=64, num_hidden_layers=1, num_attention_heads=2,
                       num_key_value_heads=1, head_dim=32, intermediate_size=128, max_position_embeddings=8)
    st = I.cfg5_model(layers=1, vocab=64, hidden=64, n_q=64, n_k=32, inter=128)
    int8_model_from_state(st, shape, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="missing"):
        int8_model_from_state({k: v for k, v in st.items() if k != "lm_head.weight"}, shape, device="cpu")
    with pytest.raises(ValueError, match="unexpected"):
        int8_model_from_state({**st, "extra": np.zeros(1)}, shape, device="cpu")
