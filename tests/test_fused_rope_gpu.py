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
