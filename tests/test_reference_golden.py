"""Pins the CPU oracle to outputs of the reference's OWN source code.

tests/golden/reference_golden.npz was produced by running the unmodified
reference files (src/pallas_flash/*.py and tests/test_paged.py helpers) under
a numpy stand-in for jax (tests/golden/make_reference_golden.py): the Pallas
forward, backward, decode, fused-RoPE and paged kernels executed grid point by
grid point, the naive ``reference_attention``, the page helpers and the model's
generate paths.  The reference's float32 arithmetic ran in float64, so the
oracle (float64) must agree to float32 rounding of those outputs.
"""

import numpy as np
import pytest

import golden_inputs as gi
from conftest import bf16_bits_to_f32
from oracle import attention_oracle as orc

ATOL = 2e-6  # float32 rounding of O(1) outputs plus float64 summation-order noise


@pytest.mark.parametrize("case", gi.FWD_CASES, ids=[c[0] for c in gi.FWD_CASES])
def test_oracle_matches_reference_forward_kernel(ref_golden, case):
    name, B, H, Hkv, Sq, Sk, D, causal, kv_len, bq, bk, seed = case
    q, k, v = gi.fwd_inputs(case)
    o = orc.reference_attention(q, k, v, causal=causal, kv_len=kv_len)
    lse = orc.attention_lse(q, k, v, causal=causal, kv_len=kv_len)
    np.testing.assert_allclose(o, ref_golden[f"fwd/{name}/o"], rtol=0, atol=ATOL)
    np.testing.assert_allclose(lse, ref_golden[f"fwd/{name}/lse"], rtol=1e-6, atol=ATOL)
    if f"fwd/{name}/naive" in ref_golden:  # reference.py's naive path agrees with its kernel
        np.testing.assert_allclose(ref_golden[f"fwd/{name}/naive"], ref_golden[f"fwd/{name}/o"],
                                   rtol=0, atol=ATOL)


@pytest.mark.parametrize("case", gi.BWD_CASES, ids=[c[0] for c in gi.BWD_CASES])
def test_oracle_vjp_matches_reference_backward_kernels(ref_golden, case):
    name, B, H, Hkv, S, D, causal, bq, bk, seed = case
    q, k, v, do = gi.bwd_inputs(case)
    got = orc.attention_vjp(q, k, v, do, causal=causal)
    for g, field in zip(got, ("dq", "dk", "dv")):
        want = ref_golden[f"bwd/{name}/{field}"]
        assert np.max(np.abs(g - want)) / np.max(np.abs(want)) < 1e-6, field


@pytest.mark.parametrize("n_kv", gi.DEC_KV)
@pytest.mark.parametrize("cache_len", gi.DEC_LENS)
def test_oracle_matches_reference_decode(ref_golden, n_kv, cache_len):
    q, kc, vc = gi.dec_inputs(n_kv)
    o = orc.reference_attention(q, kc, vc, kv_len=cache_len)
    np.testing.assert_allclose(o, ref_golden[f"dec/kv{n_kv}_len{cache_len}/o"], rtol=0, atol=ATOL)


def test_reference_decode_nan_tail_is_exactly_one(ref_golden):
    np.testing.assert_array_equal(ref_golden["dec/nan_tail/o"], np.ones((1, 2, 1, 128), np.float32))


@pytest.mark.parametrize("case", gi.ROPE_CASES, ids=[c[0] for c in gi.ROPE_CASES])
def test_oracle_matches_reference_fused_rope(ref_golden, case):
    name, B, H, Hkv, S, causal, seed = case
    q, k, v = gi.rope_inputs(case)
    cos, sin = orc.precompute_rope(S, 128, 10000.0, dtype=np.float64)
    o = orc.reference_attention(orc.apply_rope(q.astype(np.float64), cos, sin),
                                orc.apply_rope(k.astype(np.float64), cos, sin), v, causal=causal)
    # the oracle's tables are float32-argument tables (as the reference computes them on device);
    # the golden ran them in float64, so positions up to 256 leave ~3e-5 of angle difference
    np.testing.assert_allclose(o, ref_golden[f"rope/{name}/o"], rtol=0, atol=2e-4)


def test_oracle_matches_reference_rope_tables(ref_golden):
    for S, D in ((300, 128), (64, 64)):
        cos, sin = orc.precompute_rope(S, D, 10000.0)
        np.testing.assert_allclose(cos, ref_golden[f"rope/table_s{S}_d{D}/cos"], rtol=0, atol=S * 1.2e-7)
        np.testing.assert_allclose(sin, ref_golden[f"rope/table_s{S}_d{D}/sin"], rtol=0, atol=S * 1.2e-7)


def test_oracle_matches_reference_rope_decode_position(ref_golden):
    q, k, v = gi.rope_decode_inputs()
    pos = 77
    cos, sin = orc.precompute_rope(128, 128, 10000.0, dtype=np.float64)
    qr = orc.apply_rope(q.astype(np.float64), cos[pos:pos + 1], sin[pos:pos + 1])
    kr = orc.apply_rope(k.astype(np.float64), cos, sin)
    o = orc.reference_attention(qr, kr, v, kv_len=pos + 1)
    np.testing.assert_allclose(o, ref_golden["rope/decode_pos77/o"], rtol=0, atol=2e-4)


@pytest.mark.parametrize("i", range(len(gi.PAGED_CASES)))
def test_oracle_matches_reference_paged(ref_golden, i):
    B, H, Hkv, ps, lens = gi.PAGED_CASES[i]
    q, kp, vp = gi.paged_inputs(i)
    table = ref_golden[f"paged/case{i}/table"]
    o = orc.paged_attention(q, kp, vp, table, np.asarray(lens))
    np.testing.assert_allclose(o, ref_golden[f"paged/case{i}/o"], rtol=0, atol=ATOL)
    gathered = bf16_bits_to_f32(ref_golden[f"paged/case{i}/k_gathered_bf16"])
    for b, length in enumerate(lens):  # the block-table gather is bit-exact
        g = orc.gather_contiguous(kp, table[b], table.shape[1], length)
        np.testing.assert_array_equal(g, gathered[b, :, :length])


def test_oracle_matches_reference_paged_write(ref_golden):
    kseq, vseq, q = gi.paged_write_inputs()
    table = ref_golden["paged/write/table"]
    kp = np.zeros((4, 2, 32, 128), np.float32)
    vp = np.zeros_like(kp)
    for t in range(70):
        orc.paged_write(kp, vp, kseq[:, :, t:t + 1], vseq[:, :, t:t + 1], table, t)
    np.testing.assert_array_equal(kp, bf16_bits_to_f32(ref_golden["paged/write/k_pool_bf16"]))
    np.testing.assert_array_equal(vp, bf16_bits_to_f32(ref_golden["paged/write/v_pool_bf16"]))
    o = orc.paged_attention(q, kp, vp, table[None], np.asarray([70]))
    np.testing.assert_allclose(o, ref_golden["paged/write/o"], rtol=0, atol=ATOL)


def test_oracle_matches_reference_model_blocks(ref_golden):
    x, w = gi.randn((2, 5, 64), 700), gi.randn((64,), 701)
    np.testing.assert_allclose(orc.rms_norm(x, w, 1e-5), ref_golden["model/rms/y"], rtol=1e-5, atol=1e-6)
    cos, sin = orc.precompute_rope(64, 64, 10000.0, dtype=np.float64)
    np.testing.assert_allclose(orc.apply_rope(gi.randn((2, 3, 64, 64), 702).astype(np.float64), cos, sin),
                               ref_golden["model/rope/y"], rtol=0, atol=2e-5)


class _Cfg:
    def __init__(self, case):
        name, H, Hkv, hd, ffn, nl, prompt, n_new, window, seed = case
        self.vocab_size, self.dim, self.n_layers, self.n_heads = 64, H * hd, nl, H
        self.n_kv_heads, self.head_dim, self.ffn_hidden = Hkv, hd, ffn
        self.rope_theta, self.rms_norm_eps = 10000.0, 1e-5


@pytest.mark.parametrize("case", gi.MODEL_CASES, ids=[c[0] for c in gi.MODEL_CASES])
def test_oracle_model_matches_reference_logits_and_tokens(ref_golden, case):
    name, H, Hkv, hd, ffn, nl, prompt, n_new, window, seed = case
    cfg = _Cfg(case)
    params = gi.model_params(case)
    pr = np.asarray(prompt)
    logits = orc.tiny_llama_forward(params, pr, cfg)
    np.testing.assert_allclose(logits, ref_golden[f"model/{name}/logits"], rtol=0, atol=2e-4)
    # greedy decoding through the oracle reproduces the reference's generate_cached tokens
    seq = pr
    for _ in range(n_new):
        nxt = np.argmax(orc.tiny_llama_forward(params, seq, cfg)[:, -1, :], axis=-1)
        seq = np.concatenate([seq, nxt[:, None]], axis=1)
    np.testing.assert_array_equal(seq, ref_golden[f"model/{name}/tokens_cached"])
    assert float(ref_golden[f"model/{name}/margin_min"][0]) > 5e-3
    # the oracle's cached and ring-cache loops give the reference's generate_cached /
    # generate_streaming tokens
    np.testing.assert_array_equal(orc.tiny_llama_generate(params, pr, n_new, cfg),
                                  ref_golden[f"model/{name}/tokens_cached"])
    np.testing.assert_array_equal(orc.tiny_llama_generate(params, pr, n_new, cfg, window=window),
                                  ref_golden[f"model/{name}/tokens_stream"])


def test_reference_ring_kv_len(ref_golden):
    want = [orc.ring_kv_len(t, c) for t, c in ((3, 8), (8, 8), (50, 8), (1, 8))]
    np.testing.assert_array_equal(ref_golden["model/ring_kv_len"], want)
