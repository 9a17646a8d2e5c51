"""Fixed-cache decode on the GPU (port of the reference's tests/test_decode.py)."""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from oracle import attention_oracle as orc
from conftest import randn, to_dev, to_np, widen

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_kv_heads", [4, 2, 1])
@pytest.mark.parametrize("cache_len", [1, 5, 130, 256])
def test_decode_matches_reference(n_kv_heads, cache_len):
    q, k, v = randn((1, 4, 1, 128), 1), randn((1, n_kv_heads, 256, 128), 2), randn((1, n_kv_heads, 256, 128), 3)
    out = pf.flash_attention_decode(to_dev(q), to_dev(k), to_dev(v), cache_len, interpret=True)
    ref = orc.reference_attention(q, k[:, :, :cache_len], v[:, :, :cache_len])
    assert out.shape == (1, 4, 1, 128)
    assert np.max(np.abs(to_np(out) - ref)) < 2e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_decode_dtypes_and_head_dims(dtype, D):
    B, H, Hkv, C = 3, 8, 2, 1000
    q, k, v = randn((B, H, 1, D), 4), randn((B, Hkv, C, D), 5), randn((B, Hkv, C, D), 6)
    tq, tk, tv = (to_dev(x, dtype) for x in (q, k, v))
    for cache_len in (1, 31, 33, 777, 1000):
        out = pf.flash_attention_decode(tq, tk, tv, cache_len)
        ref = orc.reference_attention(widen(tq), widen(tk)[:, :, :cache_len], widen(tv)[:, :, :cache_len])
        tol = 2e-3 if dtype == torch.float32 else 2e-2
        assert np.max(np.abs(to_np(out) - ref)) < tol, cache_len


def test_decode_ignores_unwritten_slots():
    filled = 8
    k = torch.cat([torch.ones((1, 2, filled, 128)), torch.full((1, 2, 120, 128), float("nan"))], dim=2).cuda()
    q = torch.ones((1, 2, 1, 128), device="cuda")
    out = pf.flash_attention_decode(q, k, k, filled, interpret=True)
    assert torch.isfinite(out).all()
    assert torch.allclose(out, torch.ones_like(out), atol=1e-5)


def test_decode_long_split_kv():
    """Many splits (capacity 32768, GQA 4): combine across splits and warps."""
    B, H, Hkv, C, D = 2, 8, 2, 32768, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    tq = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    tk = torch.randn((B, Hkv, C, D), device="cuda", generator=g).to(torch.bfloat16)
    tv = torch.randn((B, Hkv, C, D), device="cuda", generator=g).to(torch.bfloat16)
    for cache_len in (32768, 20001, 4097):
        out = pf.flash_attention_decode(tq, tk, tv, cache_len)
        ref = orc.reference_attention(widen(tq), widen(tk)[:, :, :cache_len], widen(tv)[:, :, :cache_len])
        assert np.max(np.abs(to_np(out) - ref)) < 2e-2


def test_decode_odd_head_dim_falls_back_to_general_kernel():
    q, k, v = randn((1, 2, 1, 48), 1), randn((1, 1, 64, 48), 2), randn((1, 1, 64, 48), 3)
    out = pf.flash_attention_decode(to_dev(q), to_dev(k), to_dev(v), 40)
    assert np.max(np.abs(to_np(out) - orc.reference_attention(q, k[:, :, :40], v[:, :, :40]))) < 2e-3


def _tiny_cfg(n_heads=2, n_kv_heads=0):
    return pf.ModelConfig(vocab_size=64, dim=n_heads * 128, n_layers=2, n_heads=n_heads,
                          n_kv_heads=n_kv_heads, head_dim=128, ffn_hidden=512, max_seq_len=128)


def test_init_kv_cache_shapes():
    cfg = _tiny_cfg(n_heads=4, n_kv_heads=2)
    cache = pf.init_kv_cache(cfg, batch=2, cache_size=64)
    assert len(cache) == cfg.n_layers
    for layer in cache:
        assert layer["k"].shape == (2, cfg.n_kv_heads, 64, cfg.head_dim)
        assert layer["v"].shape == layer["k"].shape


def test_cache_capacity_is_fixed_across_steps():
    cfg = _tiny_cfg()
    params = pf.init_params(0, cfg)
    _, cache = pf.prefill(params, torch.tensor([[1, 2, 3]], device="cuda"), cfg, cache_size=16)
    assert cache[0]["k"].shape[2] == 16
    token = torch.tensor([[4]], device="cuda")
    for pos in (3, 4, 5):
        _, cache = pf.decode_step(params, token, cache, pos, cfg)
        assert cache[0]["k"].shape[2] == 16


def test_prefill_rejects_too_small_cache():
    cfg = _tiny_cfg()
    params = pf.init_params(0, cfg)
    with pytest.raises(ValueError):
        pf.prefill(params, torch.arange(8, device="cuda").reshape(1, 8), cfg, cache_size=4)


def test_decode_step_rejects_overflow():
    cfg = _tiny_cfg()
    params = pf.init_params(0, cfg)
    _, cache = pf.prefill(params, torch.tensor([[1, 2]], device="cuda"), cfg, cache_size=4)
    with pytest.raises(ValueError):
        pf.decode_step(params, torch.tensor([[3]], device="cuda"), cache, 4, cfg)


@pytest.mark.parametrize("G", [1, 3, 16, 32])
def test_decode_head_groups_bf16(G):
    """Query-head groups from MHA to 32 q heads per kv head (head chunks of 16 on the tensor-core path)."""
    B, Hkv, C, D = 2, 2, 300, 128
    q, k, v = randn((B, G * Hkv, 1, D), 7), randn((B, Hkv, C, D), 8), randn((B, Hkv, C, D), 9)
    tq, tk, tv = (to_dev(x, torch.bfloat16) for x in (q, k, v))
    out = pf.flash_attention_decode(tq, tk, tv, 257)
    ref = orc.reference_attention(widen(tq), widen(tk)[:, :, :257], widen(tv)[:, :, :257])
    assert np.max(np.abs(to_np(out) - ref)) < 2e-2


def test_decode_nan_tail_bf16():
    filled = 37
    k = torch.cat([torch.ones((2, 2, filled, 64)), torch.full((2, 2, 91, 64), float("nan"))], dim=2)
    k = k.to(torch.bfloat16).cuda()
    q = torch.ones((2, 8, 1, 64), dtype=torch.bfloat16, device="cuda")
    out = pf.flash_attention_decode(q, k, k, filled)
    assert torch.isfinite(out.float()).all()
    assert torch.allclose(out.float(), torch.ones_like(out, dtype=torch.float32), atol=1e-5)
