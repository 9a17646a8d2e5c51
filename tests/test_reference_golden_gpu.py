"""The sm_100a kernels against outputs of the reference's OWN source code.

Golden outputs: tests/golden/reference_golden.npz, made by executing the
unmodified reference files (Pallas kernels run grid point by grid point under
a numpy stand-in for jax; tests/golden/make_reference_golden.py).  Inputs are
rebuilt bit-identically by tests/golden/golden_inputs.py.

Tolerances are the ones the task fixes for this path: max abs error <= 2e-2
for bf16 inputs, <= 1e-4 relative for fp32; page-table indexing bit-exact;
greedy tokens identical.
"""

import numpy as np
import pytest
import torch

import golden_inputs as gi
import pallas_flash as pf
from conftest import bf16_bits_to_f32

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2
F32_REL = 1e-4


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dtype)


def host(t):
    return t.detach().double().cpu().numpy()


def rel(a, b):
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", gi.FWD_CASES, ids=[c[0] for c in gi.FWD_CASES])
def test_forward_and_lse_match_reference_kernel(ref_golden, case, dtype):
    name, B, H, Hkv, Sq, Sk, D, causal, kv_len, bq, bk, seed = case
    q, k, v = (dev(x, dtype) for x in gi.fwd_inputs(case))
    o, lse = pf.flash_attention_with_lse(q, k, v, causal=causal, kv_len=kv_len)
    want_o, want_lse = ref_golden[f"fwd/{name}/o"], ref_golden[f"fwd/{name}/lse"]
    if dtype == torch.float32:
        assert rel(host(o), want_o) < F32_REL
        assert rel(host(lse), want_lse) < F32_REL
    else:
        assert np.max(np.abs(host(o) - want_o)) < BF16_ATOL
        assert np.max(np.abs(host(lse) - want_lse)) < BF16_ATOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", gi.BWD_CASES, ids=[c[0] for c in gi.BWD_CASES])
def test_gradients_match_reference_backward_kernels(ref_golden, case, dtype):
    name, B, H, Hkv, S, D, causal, bq, bk, seed = case
    q, k, v, do = gi.bwd_inputs(case)
    qt, kt, vt = (dev(x, dtype).requires_grad_(True) for x in (q, k, v))
    out = pf.flash_attention(qt, kt, vt, causal=causal, block_q=bq, block_k=bk)
    out.backward(dev(do, dtype))
    for t, field in ((qt, "dq"), (kt, "dk"), (vt, "dv")):
        want = ref_golden[f"bwd/{name}/{field}"]
        got = host(t.grad)
        if dtype == torch.float32:
            assert rel(got, want) < F32_REL, field
        else:  # the reference's bf16 gradients are cast from f32 too; errors scale with |grad|
            assert np.max(np.abs(got - want)) < BF16_ATOL * max(1.0, float(np.max(np.abs(want)))), field


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("n_kv", gi.DEC_KV)
def test_decode_matches_reference(ref_golden, n_kv, dtype):
    q, kc, vc = (dev(x, dtype) for x in gi.dec_inputs(n_kv))
    for cache_len in gi.DEC_LENS:
        o = host(pf.flash_attention_decode(q, kc, vc, cache_len))
        want = ref_golden[f"dec/kv{n_kv}_len{cache_len}/o"]
        if dtype == torch.float32:
            assert rel(o, want) < F32_REL, cache_len
        else:
            assert np.max(np.abs(o - want)) < BF16_ATOL, cache_len


def test_decode_nan_tail_matches_reference_known_answer(ref_golden):
    k = torch.cat([torch.ones((1, 2, 8, 128)), torch.full((1, 2, 120, 128), float("nan"))], dim=2).cuda()
    o = pf.flash_attention_decode(torch.ones((1, 2, 1, 128), device="cuda"), k, k, 8)
    np.testing.assert_allclose(host(o), ref_golden["dec/nan_tail/o"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", gi.ROPE_CASES, ids=[c[0] for c in gi.ROPE_CASES])
def test_fused_rope_matches_reference_kernel(ref_golden, case, dtype):
    name, B, H, Hkv, S, causal, seed = case
    q, k, v = (dev(x, dtype) for x in gi.rope_inputs(case))
    cos, sin = pf.precompute_rope(S, 128, 10000.0, device="cuda")
    o = host(pf.flash_attention_rope(q, k, v, cos, sin, causal=causal))
    want = ref_golden[f"rope/{name}/o"]
    if dtype == torch.float32:  # float32 tables vs the golden's float64 ones: angle error ~S*6e-8
        assert np.max(np.abs(o - want)) < 5e-4
    else:
        assert np.max(np.abs(o - want)) < BF16_ATOL


def test_rope_tables_match_reference(ref_golden):
    for S, D in ((300, 128), (64, 64)):
        cos, sin = pf.precompute_rope(S, D, 10000.0, device="cuda")
        np.testing.assert_allclose(host(cos), ref_golden[f"rope/table_s{S}_d{D}/cos"], rtol=0, atol=S * 1.2e-7)
        np.testing.assert_allclose(host(sin), ref_golden[f"rope/table_s{S}_d{D}/sin"], rtol=0, atol=S * 1.2e-7)


def test_fused_rope_decode_position_matches_reference(ref_golden):
    q, k, v = (dev(x, torch.bfloat16) for x in gi.rope_decode_inputs())
    cos, sin = pf.precompute_rope(128, 128, 10000.0, device="cuda")
    o = pf.flash_attention_rope(q, k, v, cos[77:78], sin[77:78], cos, sin, causal=False, block_q=1,
                                kv_len=78)
    assert np.max(np.abs(host(o) - ref_golden["rope/decode_pos77/o"])) < BF16_ATOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("i", range(len(gi.PAGED_CASES)))
def test_paged_decode_and_gather_match_reference(ref_golden, i, dtype):
    B, H, Hkv, ps, lens = gi.PAGED_CASES[i]
    q, kp, vp = gi.paged_inputs(i)
    table = dev(ref_golden[f"paged/case{i}/table"], torch.int32)
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    o = host(pf.paged_flash_attention(dev(q, dtype), dev(kp, dtype), dev(vp, dtype), table, lens_t))
    want = ref_golden[f"paged/case{i}/o"]
    if dtype == torch.float32:
        assert rel(o, want) < F32_REL
    else:
        assert np.max(np.abs(o - want)) < BF16_ATOL
    # block-table gather: bit-exact against the reference test's _gather_contiguous
    g = pf.gather_paged(dev(kp, dtype), table).float().cpu().numpy()
    gathered = bf16_bits_to_f32(ref_golden[f"paged/case{i}/k_gathered_bf16"])
    for b, length in enumerate(lens):
        np.testing.assert_array_equal(g[b, :, :length], gathered[b, :, :length])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_paged_write_roundtrip_matches_reference(ref_golden, dtype):
    kseq, vseq, q = gi.paged_write_inputs()
    table = torch.tensor(ref_golden["paged/write/table"], dtype=torch.int32, device="cuda")
    kp, vp = pf.init_paged_cache(4, 2, 32, 128, dtype=dtype, device="cuda")
    ks, vs = dev(kseq, dtype), dev(vseq, dtype)
    for t in range(70):
        kp, vp = pf.write_to_paged_cache(kp, vp, ks[:, :, t:t + 1], vs[:, :, t:t + 1], table, t)
    np.testing.assert_array_equal(kp.float().cpu().numpy(), bf16_bits_to_f32(ref_golden["paged/write/k_pool_bf16"]))
    np.testing.assert_array_equal(vp.float().cpu().numpy(), bf16_bits_to_f32(ref_golden["paged/write/v_pool_bf16"]))
    o = host(pf.paged_flash_attention(dev(q, dtype), kp, vp, table[None],
                                      torch.tensor([70], dtype=torch.int32, device="cuda")))
    assert np.max(np.abs(o - ref_golden["paged/write/o"])) < (1e-4 if dtype == torch.float32 else BF16_ATOL)


def test_model_blocks_match_reference(ref_golden):
    x, w = dev(gi.randn((2, 5, 64), 700)), dev(gi.randn((64,), 701))
    assert np.max(np.abs(host(pf.rms_norm(x, w, 1e-5)) - ref_golden["model/rms/y"])) < 1e-5
    cos, sin = pf.precompute_rope(64, 64, 10000.0, device="cuda")
    y = host(pf.apply_rope(dev(gi.randn((2, 3, 64, 64), 702)), cos, sin))
    assert np.max(np.abs(y - ref_golden["model/rope/y"])) < 2e-5
    xs = dev(gi.randn((3, 64), 703))
    wg, wu, wd = (dev(gi.randn((64, 96), 704) * 0.125), dev(gi.randn((64, 96), 705) * 0.125),
                  dev(gi.randn((96, 64), 706) * 0.125))
    assert rel(host(pf.swiglu_mlp(xs, wg, wu, wd)), ref_golden["model/mlp/y"]) < F32_REL


def _params(case):
    p = gi.model_params(case)
    return {k: ([{a: dev(b) for a, b in lay.items()} for lay in v] if k == "layers" else dev(v))
            for k, v in p.items()}


@pytest.mark.parametrize("case", gi.MODEL_CASES, ids=[c[0] for c in gi.MODEL_CASES])
def test_generation_tokens_match_reference(ref_golden, case):
    """fp32 greedy tokens of forward / generate_cached / generate_streaming == the reference's."""
    name, H, Hkv, hd, ffn, nl, prompt, n_new, window, seed = case
    cfg = pf.ModelConfig(vocab_size=64, dim=H * hd, n_layers=nl, n_heads=H, n_kv_heads=Hkv,
                         head_dim=hd, ffn_hidden=ffn, max_seq_len=256)
    params = _params(case)
    pr = torch.tensor(prompt, dtype=torch.int64, device="cuda")
    logits = host(pf.forward(params, pr, cfg))
    assert np.max(np.abs(logits - ref_golden[f"model/{name}/logits"])) < 2e-3
    cached = pf.generate_cached(params, pr, n_new, cfg).cpu().numpy()
    np.testing.assert_array_equal(cached, ref_golden[f"model/{name}/tokens_cached"])
    stream = pf.generate_streaming(params, pr, n_new, cfg, window=window).cpu().numpy()
    np.testing.assert_array_equal(stream, ref_golden[f"model/{name}/tokens_stream"])
    loop = pf.generate_streaming(params, pr, n_new, cfg, window=window, use_graph=False).cpu().numpy()
    np.testing.assert_array_equal(loop, ref_golden[f"model/{name}/tokens_stream"])
