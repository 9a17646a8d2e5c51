"""Fused-RoPE forward on the GPU (port of the reference's tests/test_fused_rope.py)."""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from oracle import attention_oracle as orc
from conftest import randn, to_dev, to_np, widen

pytestmark = pytest.mark.gpu
THETA = 10000.0


def inputs(H, Hkv, S, D=128, seed=0):
    return randn((1, H, S, D), seed), randn((1, Hkv, S, D), seed + 1), randn((1, Hkv, S, D), seed + 2)


def tables(n, D=128):
    c, s = pf.precompute_rope(n, D, THETA, device="cuda")
    return c, s


@pytest.mark.parametrize("n_heads,n_kv_heads", [(2, 2), (4, 2), (4, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_fused_matches_unfused(n_heads, n_kv_heads, causal):
    q, k, v = inputs(n_heads, n_kv_heads, 256)
    cos, sin = tables(256)
    tq, tk, tv = to_dev(q), to_dev(k), to_dev(v)
    fused = pf.flash_attention_rope(tq, tk, tv, cos, sin, causal=causal, interpret=True)
    unfused = pf.flash_attention(pf.apply_rope(tq, cos, sin), pf.apply_rope(tk, cos, sin), tv, causal=causal)
    assert fused.shape == q.shape
    assert float((fused - unfused).abs().max()) < 2e-3
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    ref = orc.reference_attention(orc.apply_rope(q, c, s), orc.apply_rope(k, c, s), v, causal=causal)
    assert np.max(np.abs(to_np(fused) - ref)) < 2e-3


@pytest.mark.parametrize("seq", [130, 200])
def test_fused_ragged_lengths(seq):
    q, k, v = inputs(2, 2, seq, seed=1)
    cos, sin = tables(seq)
    tq, tk, tv = to_dev(q), to_dev(k), to_dev(v)
    fused = pf.flash_attention_rope(tq, tk, tv, cos, sin, causal=True)
    unfused = pf.flash_attention(pf.apply_rope(tq, cos, sin), pf.apply_rope(tk, cos, sin), tv, causal=True)
    assert float((fused - unfused).abs().max()) < 2e-3


def test_fused_decode_shape_separate_tables():
    pos, cache = 37, 256
    q, k, v = randn((1, 2, 1, 128), 2), randn((1, 2, cache, 128), 3), randn((1, 2, cache, 128), 4)
    cos, sin = tables(cache)
    tq, tk, tv = to_dev(q), to_dev(k), to_dev(v)
    fused = pf.flash_attention_rope(tq, tk, tv, cos[pos:pos + 1], sin[pos:pos + 1], cos, sin,
                                    causal=False, block_q=1, kv_len=pos + 1)
    unfused = pf.flash_attention(pf.apply_rope(tq, cos[pos:pos + 1], sin[pos:pos + 1]),
                                 pf.apply_rope(tk, cos, sin), tv, causal=False, kv_len=pos + 1)
    assert float((fused - unfused).abs().max()) < 2e-3


@pytest.mark.parametrize("D", [64, 128])
def test_fused_bfloat16(D):
    q, k, v = inputs(4, 2, 384, D=D, seed=3)
    cos, sin = tables(384, D)
    tq, tk, tv = (to_dev(x, torch.bfloat16) for x in (q, k, v))
    out = pf.flash_attention_rope(tq, tk, tv, cos, sin, causal=True)
    assert out.dtype == torch.bfloat16
    assert torch.isfinite(out.float()).all()
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    ref = orc.reference_attention(orc.apply_rope(widen(tq), c, s), orc.apply_rope(widen(tk), c, s), widen(tv), causal=True)
    assert np.max(np.abs(to_np(out) - ref)) < 2e-2


def test_fused_rejects_bad_table_shape():
    q, k, v = inputs(2, 2, 128, seed=4)
    cos, sin = tables(64)
    with pytest.raises(ValueError):
        pf.flash_attention_rope(to_dev(q), to_dev(k), to_dev(v), cos, sin)


def test_fused_requires_k_tables_when_lengths_differ():
    q = to_dev(randn((1, 2, 1, 128), 5))
    k = to_dev(randn((1, 2, 128, 128), 6))
    cos, sin = tables(1)
    with pytest.raises(ValueError):
        pf.flash_attention_rope(q, k, k, cos, sin, block_q=1)


@pytest.mark.parametrize("H,Hkv,Sq,Sk,D,causal,kv_len", [
    (4, 2, 256, 256, 128, True, None),
    (4, 1, 200, 200, 128, False, None),
    (8, 2, 130, 130, 64, True, None),
    (2, 2, 1, 256, 128, False, 38),     # decode shape: query at position 37, separate tables
    (4, 2, 300, 700, 64, True, 650),
])
@pytest.mark.parametrize("tdt", [torch.float32, torch.bfloat16])
def test_fused_tensor_core_path(H, Hkv, Sq, Sk, D, causal, kv_len, tdt):
    q, k, v = randn((2, H, Sq, D), 40), randn((2, Hkv, Sk, D), 41), randn((2, Hkv, Sk, D), 42)
    cos, sin = tables(max(Sq, Sk), D)
    pos0 = 37 if Sq == 1 else 0
    qc, qs = cos[pos0:pos0 + Sq].to(tdt), sin[pos0:pos0 + Sq].to(tdt)
    kc, ks = cos[:Sk].to(tdt), sin[:Sk].to(tdt)
    tq, tk, tv = (to_dev(x, torch.bfloat16) for x in (q, k, v))
    out = pf.flash_attention_rope(tq, tk, tv, qc, qs, kc, ks, causal=causal, kv_len=kv_len)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref = orc.reference_attention(orc.apply_rope(widen(tq), f(qc), f(qs)), orc.apply_rope(widen(tk), f(kc), f(ks)),
                                  widen(tv), causal=causal, kv_len=kv_len)
    assert np.max(np.abs(to_np(out) - ref)) < 2e-2


def test_c3_shape_sampled():
    """Config 3 shape at batch 1 (H32 Hkv8 S8192 D128, causal, bf16): head 5's output vs fp32 oracle."""
    g = torch.Generator(device="cuda").manual_seed(3)
    S = 8192
    tq = torch.randn((1, 32, S, 128), device="cuda", generator=g).to(torch.bfloat16)
    tk = torch.randn((1, 8, S, 128), device="cuda", generator=g).to(torch.bfloat16)
    tv = torch.randn((1, 8, S, 128), device="cuda", generator=g).to(torch.bfloat16)
    cos, sin = tables(S)
    out = pf.flash_attention_rope(tq, tk, tv, cos, sin, causal=True)
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    rows = np.array([0, 1, 4095, 8191])
    qrot = orc.apply_rope(widen(tq[:, 5:6]), c, s)[:, :, rows]
    krot = orc.apply_rope(widen(tk[:, 1:2]), c, s)
    vv = widen(tv[:, 1:2])
    for i, r in enumerate(rows):
        ref = orc.reference_attention(qrot[:, :, i:i + 1], krot[:, :, :r + 1], vv[:, :, :r + 1], dtype=np.float32)
        assert np.max(np.abs(to_np(out[:, 5:6, r:r + 1]) - ref)) < 2e-2, r


# --------------------------------------------------------------------------
# Gradient of the RoPE-fused attention (an extension: the reference's
# flash_attention_rope is forward-only, fused_rope.py:25-27).  The oracle is
# the closed-form attention VJP on the rotated inputs, mapped back through the
# transposed rotation: d x = R(-theta) d(Rx) (apply_rope with sin negated).
def _rope_grad_oracle(q, k, v, do, qc, qs, kc, ks, causal, kv_len=None):
    qr, kr = orc.apply_rope(q, qc, qs), orc.apply_rope(k, kc, ks)
    dqr, dkr, dv = orc.attention_vjp(qr, kr, v, do, causal=causal, kv_len=kv_len)
    return orc.apply_rope(dqr, qc, -qs), orc.apply_rope(dkr, kc, -ks), dv


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,S,D,causal", [(4, 2, 256, 128, True), (2, 2, 200, 64, False), (4, 1, 384, 128, True)])
def test_rope_attention_grads_match_oracle(dtype, H, Hkv, S, D, causal):
    from conftest import rel_err
    q, k, v = randn((1, H, S, D), 11), randn((1, Hkv, S, D), 12), randn((1, Hkv, S, D), 13)
    do = randn((1, H, S, D), 14)
    cos, sin = tables(S, D)
    tq, tk, tv = (to_dev(x, dtype).requires_grad_() for x in (q, k, v))
    out = pf.flash_attention_rope(tq, tk, tv, cos, sin, causal=causal)
    out.backward(to_dev(do, dtype))
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    ref = _rope_grad_oracle(widen(tq), widen(tk), widen(tv), widen(to_dev(do, dtype)), c, s, c, s, causal)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for got, want in zip((tq.grad, tk.grad, tv.grad), ref):
        assert got.dtype == dtype
        assert rel_err(to_np(got), want) < tol


def test_rope_attention_grads_cross_lengths_and_kv_len():
    """Separate query/key tables (queries at positions [Sk - Sq, Sk)) and a kv_len mask."""
    from conftest import rel_err
    Sq, Sk, kv_len = 64, 320, 300
    q, k, v = randn((2, 4, Sq, 128), 21), randn((2, 2, Sk, 128), 22), randn((2, 2, Sk, 128), 23)
    do = randn((2, 4, Sq, 128), 24)
    cos, sin = tables(Sk)
    qc, qs = cos[Sk - Sq:], sin[Sk - Sq:]
    tq, tk, tv = (to_dev(x).requires_grad_() for x in (q, k, v))
    out = pf.flash_attention_rope(tq, tk, tv, qc, qs, cos, sin, causal=False, kv_len=kv_len)
    out.backward(to_dev(do))
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    ref = _rope_grad_oracle(q, k, v, do, c[Sk - Sq:], s[Sk - Sq:], c, s, False, kv_len=kv_len)
    for got, want in zip((tq.grad, tk.grad, tv.grad), ref):
        assert rel_err(to_np(got), want) < 1e-4


def test_rope_apply_inverse_round_trip():
    x = to_dev(randn((2, 3, 50, 64), 31))
    cos, sin = tables(50, 64)
    y = pf.rope_apply(x, cos, sin)
    ref = orc.apply_rope(to_np(x), cos.cpu().numpy(), sin.cpu().numpy())
    assert np.max(np.abs(to_np(y) - ref)) < 1e-5
    back = pf.rope_apply(y, cos, sin, inverse=True)
    assert float((back - x).abs().max()) < 1e-5
