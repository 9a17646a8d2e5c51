"""pf_rows_linear (a decode step's projections with their norm / residual add /
SwiGLU activation folded in) against the unfused launches it replaces:
pf_add_rms_norm, a dtype matmul, and the residual add or pf_silu_mul
(the reference's model.py:34-38, 70-74, 120-124 as a decode step calls them).

The staged rows must equal pf_add_rms_norm's output bit for bit (same element
order and reduction), so the only difference from the unfused chain is the
summation order of the fp32 dot products: the check is an fp32 reference with
the same rounding points, to a tolerance of a few units in the last place of
the output dtype."""

import pytest
import torch

import pallas_flash as pf
from pallas_flash import _lib

pytestmark = pytest.mark.gpu

ULP = {torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}


def run(x, wt, mode, norm=None, eps=1e-5, residual=None, out=None):
    M, K = x.shape
    N = wt.shape[0] // (2 if mode == 2 else 1)
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().pf_rows_linear(
        x.data_ptr(), _lib.ptr(norm), eps, wt.data_ptr(), _lib.ptr(residual), y.data_ptr(),
        _lib.dtype_code(x.dtype), M, K, N, mode, _lib.stream_of(x)))
    return y


def reference(x, wt, mode, norm=None, eps=1e-5, residual=None):
    a = pf.add_rms_norm(x, None, norm, eps)[1] if norm is not None else x
    acc = a.float() @ wt.float().t()
    dt = x.dtype
    if mode == 0:
        return acc.to(dt)
    if mode == 1:
        return (residual.float() + acc.to(dt).float()).to(dt)
    n = wt.shape[0] // 2
    gv, uv = acc[:, :n].to(dt).float(), acc[:, n:].to(dt).float()
    s = (gv / (1.0 + torch.exp(-gv))).to(dt).float()
    return (s * uv).to(dt)


def close(y, ref, dtype, k):
    # fp32 sums of k products in a different order, then one rounding (or two)
    scale = ref.float().abs().amax().item() + 1.0
    tol = 4 * ULP[dtype] * scale
    err = (y.float() - ref.float()).abs().max().item()
    assert err <= tol, f"max error {err} > {tol}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("K,N,mode,use_norm", [
    (512, 768, 0, True),      # norm + q/k/v projection (config 5)
    (512, 512, 1, False),     # attention output projection + residual add
    (512, 1408, 2, True),     # norm + gate/up projection + SwiGLU
    (1408, 512, 1, False),    # down projection + residual add
    (512, 32000, 0, True),    # final norm + lm_head
    (64, 96, 0, False),       # small K (one unit for some warps, none for others)
    (2048, 64, 2, True),      # the largest K
])
def test_rows_linear_matches_unfused(dtype, M, K, N, mode, use_norm):
    g = torch.Generator(device="cuda").manual_seed(K + N + M + mode)
    x = torch.randn((M, K), device="cuda", generator=g).to(dtype)
    n_w = 2 * N if mode == 2 else N
    wt = (torch.randn((n_w, K), device="cuda", generator=g) / K ** 0.5).to(dtype)
    norm = (1.0 + 0.1 * torch.randn((K,), device="cuda", generator=g)).to(dtype) if use_norm else None
    res = torch.randn((M, N), device="cuda", generator=g).to(dtype) if mode == 1 else None
    y = run(x, wt, mode, norm=norm, residual=res)
    torch.cuda.synchronize()
    close(y, reference(x, wt, mode, norm=norm, residual=res), dtype, K)


def test_rows_linear_residual_in_place_and_deterministic():
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((16, 1408), device="cuda", generator=g).to(torch.bfloat16)
    wt = (torch.randn((512, 1408), device="cuda", generator=g) / 1408 ** 0.5).to(torch.bfloat16)
    res = torch.randn((16, 512), device="cuda", generator=g).to(torch.bfloat16)
    expect = run(x, wt, 1, residual=res)
    inplace = res.clone()
    run(x, wt, 1, residual=inplace, out=inplace)  # residual aliases the output
    assert torch.equal(inplace, expect)
    assert torch.equal(run(x, wt, 1, residual=res), expect)


def test_rows_linear_rejects_unsupported_shapes():
    x = torch.zeros((17, 512), device="cuda", dtype=torch.bfloat16)
    wt = torch.zeros((512, 512), device="cuda", dtype=torch.bfloat16)
    L = _lib.lib()
    y = torch.empty((17, 512), device="cuda", dtype=torch.bfloat16)
    st = L.pf_rows_linear(x.data_ptr(), None, 1e-5, wt.data_ptr(), None, y.data_ptr(), 1, 17, 512, 512, 0, None)
    assert st == _lib.PF_ERR_UNSUPPORTED  # 17 rows
    st = L.pf_rows_linear(x.data_ptr(), None, 1e-5, wt.data_ptr(), None, y.data_ptr(), 0, 16, 512, 512, 0, None)
    assert st == _lib.PF_ERR_UNSUPPORTED  # fp32
    st = L.pf_rows_linear(x.data_ptr(), None, 1e-5, wt.data_ptr(), None, y.data_ptr(), 1, 16, 512, 500, 0, None)
    assert st == _lib.PF_ERR_UNSUPPORTED  # N not a multiple of 32
    st = L.pf_rows_linear(x.data_ptr(), None, 1e-5, wt.data_ptr(), None, y.data_ptr(), 1, 16, 512, 512, 1, None)
    assert st == _lib.PF_ERR_INVALID  # mode 1 without a residual
    assert b"pf_rows_linear" in L.pf_last_error()


def test_decode_step_fused_projections_match_unfused_logits():
    """The config-5 block: a decode step through pf_rows_linear vs the same step through
    the unfused launches (norm kernel, cuBLAS matmuls, residual add, silu_mul)."""
    from pallas_flash import model as mdl

    cfg = pf.ModelConfig(vocab_size=32000, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64,
                         ffn_hidden=1408, rope_theta=10000.0, rms_norm_eps=1e-5)
    params = pf.init_params(0, cfg, dtype=torch.bfloat16)
    prompts = torch.randint(0, 32000, (16, 32), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    with torch.no_grad():
        _, cache_a = pf.prefill(params, prompts, cfg, cache_size=64)
        _, cache_b = pf.prefill(params, prompts, cfg, cache_size=64)
        tok = prompts[:, -1:]
        fused, _ = pf.decode_step(params, tok, cache_a, 32, cfg)
        orig = mdl._fused_decode_ok
        mdl._fused_decode_ok = lambda *a: False
        try:
            unfused, _ = pf.decode_step(params, tok, cache_b, 32, cfg)
        finally:
            mdl._fused_decode_ok = orig
    torch.cuda.synchronize()
    assert fused.shape == unfused.shape == (16, 1, 32000)
    err = (fused.float() - unfused.float()).abs().max().item()
    scale = unfused.float().abs().amax().item()
    assert err <= 0.03 * scale, (err, scale)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,Hkv,D,page_size", [(16, 8, 2, 64, 512), (3, 4, 4, 128, 16), (1, 2, 1, 32, 8)])
def test_rows_linear_rope_write_equals_projection_then_rope_write(dtype, B, H, Hkv, D, page_size):
    """One launch (projection + RoPE + cache write) == pf_rows_linear followed by
    pf_rope_paged_write_qkv on its output: the same rounded projection goes through the
    same rotation arithmetic, so q and both pools must be bit-identical."""
    g = torch.Generator(device="cuda").manual_seed(B * 7 + D)
    K = 512
    width = (H + 2 * Hkv) * D
    x = torch.randn((B, K), device="cuda", generator=g).to(dtype)
    wt = (torch.randn((width, K), device="cuda", generator=g) / K ** 0.5).to(dtype)
    norm = (1.0 + 0.1 * torch.randn((K,), device="cuda", generator=g)).to(dtype)
    pps = 4
    num_pages = B * pps + 3
    cos, sin = pf.precompute_rope(300, D, 10000.0, device="cuda")
    table = torch.randperm(num_pages, device="cuda", generator=g)[:B * pps].to(torch.int32).reshape(B, pps)
    pos = torch.randint(0, pps * page_size, (B,), device="cuda", generator=g).to(torch.int32)
    rpos = torch.randint(0, 300, (B,), device="cuda", generator=g).to(torch.int32)
    pools = [torch.randn((num_pages, Hkv, page_size, D), device="cuda", generator=g).to(dtype) for _ in range(2)]
    ka, va = pools[0].clone(), pools[1].clone()
    kb, vb = pools[0].clone(), pools[1].clone()
    qa = torch.empty((B, H, 1, D), device="cuda", dtype=dtype)
    L = _lib.lib()
    _lib.check(L.pf_rows_linear_rope_write(
        x.data_ptr(), norm.data_ptr(), 1e-5, wt.data_ptr(), qa.data_ptr(), ka.data_ptr(), va.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), _lib.dtype_code(cos.dtype), cos.shape[0], table.data_ptr(), pos.data_ptr(),
        rpos.data_ptr(), _lib.dtype_code(dtype), B, K, H, Hkv, num_pages, page_size, pps, D, None))
    qkv = run(x, wt, 0, norm=norm)
    qb = pf.rope_write_to_paged_cache_qkv(qkv.reshape(B, 1, width), H, kb, vb, cos, sin, table, pos, rpos)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb)
    assert torch.equal(ka, kb) and torch.equal(va, vb)
    assert not torch.equal(ka, pools[0])  # the rows were written
