"""Host-side behaviour of the Python API that needs no GPU: the reference's
ValueError rules, config validation, ring bookkeeping, and the refusal to run
on CPU tensors (there is no CPU fallback)."""

import pytest
import torch

import pallas_flash as pf


def test_gqa_requires_divisible_heads():
    q = torch.zeros((1, 6, 128, 128))
    k = v = torch.zeros((1, 4, 128, 128))
    with pytest.raises(ValueError):
        pf.flash_attention(q, k, v, interpret=True)


def test_rank_and_shape_errors():
    with pytest.raises(ValueError):
        pf.flash_attention(torch.zeros(2, 3, 4), torch.zeros(2, 3, 4), torch.zeros(2, 3, 4))
    with pytest.raises(ValueError):
        pf.flash_attention(torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 5, 8))
    with pytest.raises(ValueError):
        pf.flash_attention(torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 4, 8), kv_len=5)


def test_decode_rejects_multi_row_query():
    q = torch.zeros((1, 2, 4, 128))
    k = v = torch.zeros((1, 2, 128, 128))
    with pytest.raises(ValueError):
        pf.flash_attention_decode(q, k, v, 128, interpret=True)


def test_paged_rejects_multi_row_query():
    k_pages = v_pages = torch.zeros((4, 2, 32, 128))
    with pytest.raises(ValueError):
        pf.paged_flash_attention(torch.zeros((1, 2, 4, 128)), k_pages, v_pages,
                                 torch.zeros((1, 2), dtype=torch.int32), torch.tensor([32]))


def test_fused_rope_argument_errors():
    q = k = v = torch.zeros((1, 2, 128, 128))
    cos, sin = pf.precompute_rope(64, 128, 10000.0)
    with pytest.raises(ValueError):
        pf.flash_attention_rope(q, k, v, cos, sin, interpret=True)
    q1 = torch.zeros((1, 2, 1, 128))
    c1, s1 = pf.precompute_rope(1, 128, 10000.0)
    with pytest.raises(ValueError):
        pf.flash_attention_rope(q1, k, v, c1, s1, block_q=1, interpret=True)


def test_cpu_tensors_are_refused_not_emulated():
    q = k = v = torch.zeros((1, 2, 8, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        pf.flash_attention(q, k, v)


def test_model_config_rules():
    c = pf.ModelConfig(dim=256, n_heads=2, head_dim=128)
    assert c.n_kv_heads == 2 and c.kv_dim == 256
    with pytest.raises(ValueError):
        pf.ModelConfig(dim=300, n_heads=2, head_dim=128)
    with pytest.raises(ValueError):
        pf.ModelConfig(dim=384, n_heads=3, n_kv_heads=2, head_dim=128)
    c5 = pf.ModelConfig(vocab_size=32000, dim=512, n_layers=8, n_heads=8, n_kv_heads=2,
                        head_dim=64, ffn_hidden=1408)
    assert c5.kv_dim == 128


def test_ring_kv_len():
    assert pf.ring_kv_len(3, 8) == 3
    assert pf.ring_kv_len(8, 8) == 8
    assert pf.ring_kv_len(50, 8) == 8
    assert pf.ring_kv_len(1, 8) == 1


def test_precompute_rope_shapes():
    cos, sin = pf.precompute_rope(16, 64, 10000.0)
    assert cos.shape == (16, 64) and sin.shape == (16, 64)
    assert torch.allclose(cos[0], torch.ones(64)) and torch.allclose(sin[0], torch.zeros(64))
