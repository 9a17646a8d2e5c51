"""Pins the CPU oracle (oracle/attention_oracle.py) before it is trusted.

* against tests/golden/ fixtures (float64 torch autograd of the reference's
  naive attention, made by tests/golden/make_golden.py);
* against the reference tests' known-answer cases (uniform attention over
  all-ones values, NaN past the valid length, shared pages, key-order
  invariance, ring_kv_len table).
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from conftest import randn


def _meta(c):
    B, H, Hkv, Sq, Sk, D, causal, kv_len = (int(x) for x in c["meta"])
    return B, H, Hkv, Sq, Sk, D, bool(causal), (None if kv_len < 0 else kv_len)


@pytest.mark.parametrize("name", ["mha_noncausal", "mha_causal_ragged", "gqa_causal",
                                  "mqa_noncausal", "kvlen_decode", "custom_scale", "cross_causal"])
def test_oracle_matches_golden(golden, name):
    c = golden[name]
    _, _, _, _, _, _, causal, kv_len = _meta(c)
    scale = float(c["scale"])
    out = orc.reference_attention(c["q"], c["k"], c["v"], causal=causal, sm_scale=scale, kv_len=kv_len)
    np.testing.assert_allclose(out, c["out"], rtol=0, atol=1e-12)
    dq, dk, dv = orc.attention_vjp(c["q"], c["k"], c["v"], c["do"], causal=causal, sm_scale=scale,
                                   kv_len=kv_len)
    for got, want in ((dq, c["dq"]), (dk, c["dk"]), (dv, c["dv"])):
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-10)


def test_oracle_f32_close_to_f64(golden):
    c = golden["gqa_causal"]
    out32 = orc.reference_attention(c["q"], c["k"], c["v"], causal=True, dtype=np.float32)
    assert np.max(np.abs(out32 - c["out"])) < 1e-5


def test_known_answer_uniform_ones_with_nan_tail():
    """tests/test_decode.py:38-49 -- all-ones prefix, NaN past cache_len -> exactly 1.0."""
    k = np.concatenate([np.ones((1, 2, 8, 16)), np.full((1, 2, 20, 16), np.nan)], axis=2)
    q = np.ones((1, 2, 1, 16))
    out = orc.reference_attention(q, k, k, kv_len=8)
    assert np.all(np.isfinite(out))
    np.testing.assert_allclose(out, 1.0, atol=1e-12)


def test_known_answer_roll_invariance():
    """tests/test_streaming.py:82-103 -- attention is invariant to key order."""
    q, k, v = randn((1, 2, 1, 16), 1), randn((1, 2, 8, 16), 2), randn((1, 2, 8, 16), 3)
    a = orc.reference_attention(q, k, v)
    b = orc.reference_attention(q, np.roll(k, 3, axis=2), np.roll(v, 3, axis=2))
    np.testing.assert_allclose(a, b, atol=1e-12)


def test_known_answer_shared_pages_and_gather():
    """tests/test_paged.py:61-74 and :25-28 -- shared pages agree; gather follows the table."""
    pages = randn((8, 2, 4, 16), 5)
    table = np.array([[3, 5], [3, 5]])
    q1 = randn((1, 2, 1, 16), 6)
    q = np.concatenate([q1, q1])
    out = orc.paged_attention(q, pages, pages, table, np.array([7, 7]))
    np.testing.assert_array_equal(out[0], out[1])
    g = orc.gather_contiguous(pages, table[0], 2, 7)
    np.testing.assert_array_equal(g[:, :4], pages[3])
    np.testing.assert_array_equal(g[:, 4:7], pages[5][:, :3])


def test_paged_write_roundtrip():
    """tests/test_paged.py:94-115 -- tokens written through the table are the ones attended."""
    ps, D, n_kv, n_pages, length = 4, 8, 2, 4, 13
    kp = np.zeros((n_pages, n_kv, ps, D))
    vp = np.zeros_like(kp)
    table = np.array([0, 2, 1, 3])
    ks, vs = randn((1, n_kv, length, D), 7), randn((1, n_kv, length, D), 8)
    for pos in range(length):
        orc.paged_write(kp, vp, ks[:, :, pos:pos + 1], vs[:, :, pos:pos + 1], table, pos)
    q = randn((1, 2, 1, D), 9)
    got = orc.paged_attention(q, kp, vp, table[None], np.array([length]))
    np.testing.assert_allclose(got, orc.reference_attention(q, ks, vs), atol=1e-12)


def test_ring_helpers():
    """tests/test_streaming.py:28-32 and model.py:434-437."""
    assert [orc.ring_kv_len(t, 8) for t in (3, 8, 50, 1)] == [3, 8, 8, 1]
    np.testing.assert_array_equal(orc.ring_slots(12, 20, 8), [4, 5, 6, 7, 0, 1, 2, 3])


def test_rope_matches_torch_rotation():
    cos, sin = orc.precompute_rope(5, 8, 10000.0)
    x = randn((1, 1, 5, 8), 10)
    got = orc.apply_rope(x, cos, sin)
    tx = torch.tensor(x)
    half = 4
    rot = torch.cat([-tx[..., half:], tx[..., :half]], dim=-1)
    want = tx * torch.tensor(cos) + rot * torch.tensor(sin)
    np.testing.assert_allclose(got, want.numpy(), atol=1e-6)
    # position 0 is the identity rotation
    np.testing.assert_allclose(got[..., 0, :], x[..., 0, :], atol=1e-7)


def test_round_bf16_matches_torch():
    x = randn((1000,), 11) * 100
    want = torch.tensor(x).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(orc.round_bf16(x), want)


def test_lse_consistent_with_softmax(golden):
    c = golden["mha_causal_ragged"]
    lse = orc.attention_lse(c["q"], c["k"], c["v"], causal=True)
    s = np.einsum("bhqd,bhkd->bhqk", c["q"].astype(np.float64), c["k"].astype(np.float64)) / 4.0
    s = np.where(np.tril(np.ones(s.shape[-2:], bool)), s, -np.inf)
    np.testing.assert_allclose(lse[..., 0], np.log(np.exp(s).sum(-1)), atol=1e-10)
