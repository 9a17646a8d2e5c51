"""Tiny-LLaMA paths on the GPU (port of the reference's tests/test_model.py and
the model half of tests/test_bfloat16.py), plus logits vs the numpy oracle."""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _tiny_cfg(n_heads=2, n_kv_heads=0, head_dim=128):
    return pf.ModelConfig(vocab_size=64, dim=n_heads * head_dim, n_layers=2, n_heads=n_heads,
                          n_kv_heads=n_kv_heads, head_dim=head_dim, ffn_hidden=512, max_seq_len=256)


def test_forward_shape_and_finite():
    cfg = _tiny_cfg()
    params = pf.init_params(0, cfg)
    logits = pf.forward(params, torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]], device="cuda"), cfg)
    assert logits.shape == (1, 8, cfg.vocab_size)
    assert torch.isfinite(logits).all()


def test_forward_matches_numpy_oracle():
    cfg = _tiny_cfg(n_heads=4, n_kv_heads=2, head_dim=64)
    params = pf.init_params(3, cfg)
    tokens = torch.tensor([[1, 5, 9, 2, 60, 33, 7, 8, 9, 10, 11]], device="cuda")
    got = pf.forward(params, tokens, cfg).cpu().numpy()
    np_params = {"embed": params["embed"].cpu().numpy(), "final_norm": params["final_norm"].cpu().numpy(),
                 "lm_head": params["lm_head"].cpu().numpy(),
                 "layers": [{k: v.cpu().numpy() for k, v in l.items()} for l in params["layers"]]}
    want = orc.tiny_llama_forward(np_params, tokens.cpu().numpy(), cfg)
    assert np.max(np.abs(got - want)) < 2e-3


def test_generate_length_and_prefix():
    cfg = _tiny_cfg()
    params = pf.init_params(1, cfg)
    prompt = torch.tensor([[3, 1, 4, 1, 5]], device="cuda")
    out = pf.generate(params, prompt, max_new_tokens=6, cfg=cfg)
    assert out.shape == (1, prompt.shape[1] + 6)
    assert torch.equal(out[:, :prompt.shape[1]], prompt)


def test_generate_deterministic():
    cfg = _tiny_cfg()
    params = pf.init_params(2, cfg)
    prompt = torch.tensor([[2, 7, 1]], device="cuda")
    assert torch.equal(pf.generate(params, prompt, 4, cfg), pf.generate(params, prompt, 4, cfg))


def test_single_block_finite():
    cfg = _tiny_cfg()
    params = pf.init_params(3, cfg)
    x = torch.randn((1, 16, cfg.dim), device="cuda")
    cos, sin = pf.precompute_rope(16, cfg.head_dim, cfg.rope_theta, device="cuda")
    y = pf.decoder_block(params["layers"][0], x, cos, sin, cfg)
    assert y.shape == x.shape and torch.isfinite(y).all()


@pytest.mark.parametrize("n_heads,n_kv_heads", [(2, 2), (4, 2), (4, 1)])
def test_gqa_forward(n_heads, n_kv_heads):
    cfg = _tiny_cfg(n_heads=n_heads, n_kv_heads=n_kv_heads)
    params = pf.init_params(0, cfg)
    assert params["layers"][0]["wk"].shape == (cfg.dim, cfg.kv_dim)
    logits = pf.forward(params, torch.tensor([[1, 2, 3, 4, 5]], device="cuda"), cfg)
    assert logits.shape == (1, 5, cfg.vocab_size) and torch.isfinite(logits).all()


@pytest.mark.parametrize("n_heads,n_kv_heads", [(2, 2), (4, 2), (4, 1)])
def test_cached_matches_recompute(n_heads, n_kv_heads):
    cfg = _tiny_cfg(n_heads=n_heads, n_kv_heads=n_kv_heads)
    params = pf.init_params(5, cfg)
    prompt = torch.tensor([[5, 9, 2, 7, 1]], device="cuda")
    assert torch.equal(pf.generate(params, prompt, 8, cfg), pf.generate_cached(params, prompt, 8, cfg))


def test_bf16_model_forward_and_generate():
    cfg = pf.ModelConfig(vocab_size=64, dim=256, n_layers=2, n_heads=2, head_dim=128, ffn_hidden=512,
                         max_seq_len=128)
    params = pf.init_params(0, cfg, dtype=torch.bfloat16)
    assert params["layers"][0]["wq"].dtype == torch.bfloat16
    logits = pf.forward(params, torch.tensor([[1, 2, 3, 4]], device="cuda"), cfg)
    assert torch.isfinite(logits.float()).all()
    out = pf.generate_cached(params, torch.tensor([[1, 2, 3]], device="cuda"), max_new_tokens=4, cfg=cfg)
    assert out.shape == (1, 7)


def test_c5_config_generate_cached_and_streaming():
    """BASELINE config 5 architecture (bf16, head_dim 64, GQA 8/2) on a short run."""
    cfg = pf.ModelConfig(vocab_size=32000, dim=512, n_layers=8, n_heads=8, n_kv_heads=2, head_dim=64,
                         ffn_hidden=1408, rope_theta=10000.0, rms_norm_eps=1e-5)
    params = pf.init_params(0, cfg, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(0)
    prompts = torch.randint(0, 32000, (16, 128), device="cuda", generator=g)
    cached = pf.generate_cached(params, prompts, 16, cfg, cache_size=512)
    assert cached.shape == (16, 144) and torch.equal(cached[:, :128], prompts)
    streamed = pf.generate_streaming(params, prompts, 16, cfg, window=512)
    assert torch.equal(streamed, cached)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("head_dim,cache_size", [(128, 32), (64, 512)])
def test_graph_decode_equals_step_loop(dtype, head_dim, cache_size):
    """generate_cached replaying one captured CUDA graph == the step-by-step loop."""
    cfg = _tiny_cfg(n_heads=4, n_kv_heads=2, head_dim=head_dim)
    params = pf.init_params(9, cfg, dtype=dtype)
    prompt = torch.tensor([[5, 9, 2, 7, 1], [3, 3, 8, 1, 0]], device="cuda")
    a = pf.generate_cached(params, prompt, 12, cfg, cache_size=cache_size, use_graph=True)
    b = pf.generate_cached(params, prompt, 12, cfg, cache_size=cache_size, use_graph=False)
    assert torch.equal(a, b)
