"""Ring-buffer cache on the GPU (port of the reference's tests/test_streaming.py)."""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from oracle import attention_oracle as orc
from conftest import randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _cfg(n_heads=2, n_kv_heads=0, head_dim=128):
    return pf.ModelConfig(vocab_size=64, dim=n_heads * head_dim, n_layers=2, n_heads=n_heads,
                          n_kv_heads=n_kv_heads, head_dim=head_dim, ffn_hidden=512, max_seq_len=256)


def test_ring_cache_shape_is_constant():
    cfg = _cfg()
    cache = pf.init_ring_cache(cfg, batch=1, capacity=16)
    assert cache[0]["k"].shape == (1, cfg.n_kv_heads, 16, cfg.head_dim)


@pytest.mark.parametrize("n_heads,n_kv_heads", [(2, 2), (4, 2)])
def test_streaming_matches_cached_when_nothing_evicted(n_heads, n_kv_heads):
    cfg = _cfg(n_heads, n_kv_heads)
    params = pf.init_params(0, cfg)
    prompt = torch.tensor([[5, 9, 2, 7, 1]], device="cuda")
    streamed = pf.generate_streaming(params, prompt, 10, cfg, window=64)
    cached = pf.generate_cached(params, prompt, 10, cfg)
    assert torch.equal(streamed, cached)


def test_streaming_runs_in_constant_memory_when_window_wraps():
    cfg = _cfg()
    params = pf.init_params(1, cfg)
    prompt = torch.tensor([[5, 9, 2, 7, 1]], device="cuda")
    window = 8
    out = pf.generate_streaming(params, prompt, 20, cfg, window=window)
    assert out.shape == (1, prompt.shape[1] + 20)
    _, cache = pf.prefill_ring(params, prompt, cfg, window)
    token = torch.tensor([[3]], device="cuda")
    for pos in range(prompt.shape[1], prompt.shape[1] + 15):
        _, cache = pf.ring_decode_step(params, token, cache, pos, cfg)
        assert cache[0]["k"].shape[2] == window


def test_prefill_ring_keeps_the_most_recent_window():
    cfg = _cfg()
    params = pf.init_params(2, cfg)
    window = 8
    prompt = (torch.arange(20, device="cuda").reshape(1, 20) % cfg.vocab_size)
    _, cache = pf.prefill_ring(params, prompt, cfg, window)
    assert cache[0]["k"].shape[2] == window
    assert bool((cache[0]["k"] != 0).any(dim=-1).all())


def test_prefill_ring_slots_match_oracle():
    """Slot pos % C holds the post-RoPE key of absolute position pos (model.py:434-449)."""
    cfg = _cfg()
    params = pf.init_params(4, cfg)
    window, seq = 8, 21
    prompt = torch.arange(seq, device="cuda").reshape(1, seq) % cfg.vocab_size
    _, ring = pf.prefill_ring(params, prompt, cfg, window)
    _, full = pf.prefill(params, prompt, cfg, cache_size=seq)
    slots = orc.ring_slots(seq - window, seq, window)
    for i, pos in enumerate(range(seq - window, seq)):
        assert torch.equal(ring[0]["k"][:, :, slots[i]], full[0]["k"][:, :, pos])


def test_ring_layout_is_permutation_invariant():
    capacity, dim = 8, 128
    q, k, v = randn((1, 2, 1, dim), 3), randn((1, 2, capacity, dim), 4), randn((1, 2, capacity, dim), 5)
    in_order = pf.flash_attention_decode(to_dev(q), to_dev(k), to_dev(v), capacity, block_k=capacity)
    rolled = pf.flash_attention_decode(to_dev(q), to_dev(np.roll(k, 3, axis=2)), to_dev(np.roll(v, 3, axis=2)),
                                       capacity, block_k=capacity)
    assert float((in_order - rolled).abs().max()) < 2e-3
    assert np.max(np.abs(to_np(in_order) - orc.reference_attention(q, k, v))) < 2e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graph_streaming_equals_step_loop_when_wrapping(dtype):
    cfg = _cfg(n_heads=4, n_kv_heads=2)
    params = pf.init_params(3, cfg, dtype=dtype)
    prompt = torch.tensor([[5, 9, 2, 7, 1, 4, 4, 6, 2, 9, 1]], device="cuda")
    a = pf.generate_streaming(params, prompt, 30, cfg, window=8, use_graph=True)
    b = pf.generate_streaming(params, prompt, 30, cfg, window=8, use_graph=False)
    assert torch.equal(a, b)
