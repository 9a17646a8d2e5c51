"""Backward parity on the GPU (port of the reference's tests/test_backward.py).

Gradients of ``sum(flash_attention(q,k,v) * cot)`` through torch.autograd vs the
oracle's closed-form VJP of the naive attention (what the reference compares
with jax.grad).  fp32 bar: relative error < 1e-4 (tests/test_backward.py:65).
"""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from oracle import attention_oracle as orc
from conftest import randn, to_dev, to_np, widen, rel_err

pytestmark = pytest.mark.gpu

CASES = [(1, 2, 2, 128), (1, 2, 2, 256), (2, 4, 4, 256), (1, 4, 2, 256), (1, 4, 1, 256), (1, 2, 2, 200)]


def inputs(B, H, Hkv, S, D, seed):
    return (randn((B, H, S, D), seed), randn((B, Hkv, S, D), seed + 1),
            randn((B, Hkv, S, D), seed + 2), randn((B, H, S, D), seed + 3))


def grads(q, k, v, cot, causal, dtype=torch.float32, **kw):
    tq, tk, tv = (to_dev(x, dtype).requires_grad_(True) for x in (q, k, v))
    out = pf.flash_attention(tq, tk, tv, causal=causal, **kw)
    (out.float() * to_dev(cot)).sum().backward()
    return tq, tk, tv, out


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_grads_match_reference(case, causal):
    B, H, Hkv, S = case
    q, k, v, cot = inputs(B, H, Hkv, S, 128, 0)
    tq, tk, tv, _ = grads(q, k, v, cot, causal)
    want = orc.attention_vjp(q, k, v, cot, causal=causal)
    for t, w in zip((tq, tk, tv), want):
        assert t.grad.shape == t.shape and t.grad.dtype == torch.float32
        g = to_np(t.grad)
        assert np.all(np.isfinite(g))
        assert rel_err(g, w) < 1e-4


@pytest.mark.parametrize("block", [(64, 64), (128, 256), (256, 128)])
def test_grads_block_sizes(block):
    q, k, v, cot = inputs(1, 2, 2, 256, 128, 3)
    tq, tk, tv, _ = grads(q, k, v, cot, True, block_q=block[0], block_k=block[1])
    for t, w in zip((tq, tk, tv), orc.attention_vjp(q, k, v, cot, causal=True)):
        assert rel_err(to_np(t.grad), w) < 1e-4


def test_grads_bfloat16_finite_and_close():
    q, k, v, cot = inputs(1, 4, 2, 384, 128, 4)
    tq, tk, tv, _ = grads(q, k, v, cot, True, dtype=torch.bfloat16)
    want = orc.attention_vjp(widen(tq), widen(tk), widen(tv), cot, causal=True)
    for t, w in zip((tq, tk, tv), want):
        assert t.grad.dtype == torch.bfloat16
        g = to_np(t.grad)
        assert np.all(np.isfinite(g))
        assert rel_err(g, w) < 2e-2


def test_kv_len_and_cross_lengths():
    q, k, v = randn((1, 4, 90, 64), 5), randn((1, 2, 160, 64), 6), randn((1, 2, 160, 64), 7)
    cot = randn((1, 4, 90, 64), 8)
    tq, tk, tv = (to_dev(x).requires_grad_(True) for x in (q, k, v))
    (pf.flash_attention(tq, tk, tv, causal=True, kv_len=100) * to_dev(cot)).sum().backward()
    want = orc.attention_vjp(q, k, v, cot, causal=True, kv_len=100)
    for t, w in zip((tq, tk, tv), want):
        assert rel_err(to_np(t.grad), w) < 1e-4
    assert float(tk.grad[:, :, 100:].abs().max()) == 0.0


def test_value_and_grad_composes():
    """tests/test_backward.py:94-105: loss value and finite grads."""
    q, k, v, cot = inputs(1, 2, 2, 128, 128, 5)
    tq, tk, tv, out = grads(q, k, v, cot, True)
    value = float((out * to_dev(cot)).sum())
    ref = float((orc.reference_attention(q, k, v, causal=True) * cot).sum())
    assert abs(value - ref) <= 1e-4 + 1e-4 * abs(ref)
    assert all(torch.isfinite(t.grad).all() for t in (tq, tk, tv))


def test_golden_grads_on_gpu(golden):
    for name, c in golden.items():
        B, H, Hkv, Sq, Sk, D, causal, kv_len = (int(x) for x in c["meta"])
        tq, tk, tv = (to_dev(c[n]).requires_grad_(True) for n in ("q", "k", "v"))
        out = pf.flash_attention(tq, tk, tv, causal=bool(causal), sm_scale=float(c["scale"]),
                                 kv_len=None if kv_len < 0 else kv_len)
        (out * to_dev(c["do"])).sum().backward()
        for t, n in ((tq, "dq"), (tk, "dk"), (tv, "dv")):
            assert rel_err(to_np(t.grad), c[n]) < 1e-4, (name, n)


# ---------------------------------------------------------------- tensor-core path
TC_CASES = [
    # (B, H, Hkv, Sq, Sk, D, causal, kv_len)
    (1, 2, 2, 128, 128, 128, True, None),
    (2, 4, 2, 256, 256, 128, False, None),
    (1, 4, 1, 200, 200, 128, True, None),
    (1, 8, 2, 1000, 1000, 64, True, None),
    (2, 4, 4, 64, 64, 64, False, None),
    (1, 4, 2, 300, 700, 128, True, None),
    (1, 4, 2, 90, 640, 128, False, 333),
    (1, 2, 1, 257, 257, 64, True, 130),
]


@pytest.mark.parametrize("case", TC_CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_grads(case, dtype):
    B, H, Hkv, Sq, Sk, D, causal, kv_len = case
    q, k, v = randn((B, H, Sq, D), 21), randn((B, Hkv, Sk, D), 22), randn((B, Hkv, Sk, D), 23)
    cot = randn((B, H, Sq, D), 24)
    tq, tk, tv = (to_dev(x, dtype).requires_grad_(True) for x in (q, k, v))
    out = pf.flash_attention(tq, tk, tv, causal=causal, kv_len=kv_len)
    out.backward(to_dev(cot, dtype))
    want = orc.attention_vjp(widen(tq), widen(tk), widen(tv), widen(to_dev(cot, dtype)), causal=causal,
                             kv_len=kv_len)
    for t, w, name in zip((tq, tk, tv), want, ("dq", "dk", "dv")):
        assert t.grad.dtype == dtype
        g = to_np(t.grad)
        assert np.all(np.isfinite(g)), name
        assert rel_err(g, w) < 2e-2, (name, rel_err(g, w))
    if kv_len is not None:
        assert float(tk.grad[:, :, kv_len:].float().abs().max()) == 0.0


def test_tensor_core_grads_c2_shape_sampled():
    """Config 2 shape at reduced batch (B1 H32 Hkv8 S4096 D128, causal): a few (head, row) slices."""
    g = torch.Generator(device="cuda").manual_seed(7)
    shp_q, shp_k = (1, 32, 4096, 128), (1, 8, 4096, 128)
    tq = torch.randn(shp_q, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    tk = torch.randn(shp_k, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    tv = torch.randn(shp_k, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    do = torch.randn(shp_q, device="cuda", generator=g).to(torch.bfloat16)
    pf.flash_attention(tq, tk, tv, causal=True).backward(do)
    # kv head 3 (q heads 12..15), full-precision oracle on that group only
    sl = slice(12, 16)
    want = orc.attention_vjp(widen(tq[:, sl]), widen(tk[:, 3:4]), widen(tv[:, 3:4]), widen(do[:, sl]),
                             causal=True, dtype=np.float32)
    for t, w, name in ((tq.grad[:, sl], want[0], "dq"), (tk.grad[:, 3:4], want[1], "dk"),
                       (tv.grad[:, 3:4], want[2], "dv")):
        assert rel_err(to_np(t), w) < 2e-2, name


@pytest.mark.parametrize("B,H,Hkv,S,causal,kv_len", [(4, 8, 2, 512, True, None), (3, 6, 3, 384, False, 301),
                                                   (9, 4, 1, 256, True, None)])
def test_ds_spill_path_matches_recompute_path(B, H, Hkv, S, causal, kv_len):
    """pf_bwd with its full workspace (dK/dV spills dS; dQ is a GEMM over the spill,
    pipelined over chunks of (batch, kv-head) units on two streams) against pf_bwd with a
    delta-only workspace (dQ recomputes S and dP): dK/dV bit-identical (the same kernel),
    dQ within bf16 summation-order noise; both against the oracle."""
    from pallas_flash import _lib
    from pallas_flash.flash_attention import _fwd
    D = 128
    q, k, v, do = (to_dev(x, torch.bfloat16) for x in inputs(B, H, Hkv, S, D, 11))
    scale = 1.0 / np.sqrt(D)
    kl = S if kv_len is None else kv_len
    out, lse = _fwd(q, k, v, causal, scale, kl, True)
    L = _lib.lib()
    full = L.pf_bwd_workspace_size(1, B, H, Hkv, S, S, D, int(causal), kl)
    ws = torch.empty(full, dtype=torch.uint8, device="cuda")
    res = []
    for nbytes in (full, B * H * S * 4):
        g = [torch.empty_like(t) for t in (q, k, v)]
        _lib.check(L.pf_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), do.data_ptr(),
                            lse.data_ptr(), g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr(), 1, B, H, Hkv, S, S,
                            D, int(causal), scale, kl, ws.data_ptr(), nbytes, _lib.stream_of(q)))
        torch.cuda.synchronize()
        res.append(g)
    assert _lib.device_status(reset=True) == 0
    if L.pf_bwd_head_parts(B, H, Hkv, S) == 1:
        assert torch.equal(res[0][1], res[1][1]) and torch.equal(res[0][2], res[1][2])
    else:  # the full workspace also splits the q heads: f32 partials summed in another order
        for a, b in ((res[0][1], res[1][1]), (res[0][2], res[1][2])):
            assert float((a.float() - b.float()).abs().max()) <= 1e-2 * max(1.0, float(b.float().abs().max()))
    dq_s, dq_r = to_np(res[0][0]), to_np(res[1][0])
    assert np.max(np.abs(dq_s - dq_r)) <= 2e-2 * max(1.0, float(np.max(np.abs(dq_r))))
    rq, rk, rv = orc.attention_vjp(widen(q), widen(k), widen(v), widen(do), causal=causal, kv_len=kv_len)
    for got, want in ((dq_s, rq), (to_np(res[0][1]), rk), (to_np(res[0][2]), rv)):
        assert rel_err(got, want) < 2e-2


@pytest.mark.parametrize("B,H,Hkv,S,causal,kv_len", [(1, 16, 4, 4096, True, None), (1, 8, 2, 384, False, 301),
                                                   (2, 8, 1, 640, True, None)])
def test_head_split_matches_unsplit(B, H, Hkv, S, causal, kv_len):
    """Small problems (fewer key-tile CTAs than SMs) split each kv group's q heads over
    several dK/dV CTAs with f32 partial sums: against the same call without room for the
    partials, dQ is bit-identical (same dS tiles, same GEMM), dK/dV within the rounding of
    a different f32 summation order; both against the oracle; no device status flags."""
    from pallas_flash import _lib
    from pallas_flash.flash_attention import _fwd
    D = 128
    L = _lib.lib()
    parts = L.pf_bwd_head_parts(B, H, Hkv, S)
    assert parts > 1
    q, k, v, do = (to_dev(x, torch.bfloat16) for x in inputs(B, H, Hkv, S, D, 5))
    scale = 1.0 / np.sqrt(D)
    kl = S if kv_len is None else kv_len
    out, lse = _fwd(q, k, v, causal, scale, kl, True)
    full = L.pf_bwd_workspace_size(1, B, H, Hkv, S, S, D, int(causal), kl)
    part_bytes = 2 * parts * B * Hkv * S * D * 4
    ws = torch.empty(full, dtype=torch.uint8, device="cuda")
    _lib.device_status(reset=True)
    res = []
    for nbytes in (full, full - part_bytes):
        g = [torch.empty_like(t) for t in (q, k, v)]
        _lib.check(L.pf_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), do.data_ptr(),
                            lse.data_ptr(), g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr(), 1, B, H, Hkv, S, S,
                            D, int(causal), scale, kl, ws.data_ptr(), nbytes, _lib.stream_of(q)))
        torch.cuda.synchronize()
        res.append(g)
    assert _lib.device_status(reset=True) == 0
    assert torch.equal(res[0][0], res[1][0])
    for a, b in ((res[0][1], res[1][1]), (res[0][2], res[1][2])):
        assert float((a.float() - b.float()).abs().max()) <= 1e-2 * max(1.0, float(b.float().abs().max()))
    if S <= 1024:
        rq, rk, rv = orc.attention_vjp(widen(q), widen(k), widen(v), widen(do), causal=causal, kv_len=kv_len)
        for got, want in ((res[0][0], rq), (res[0][1], rk), (res[0][2], rv)):
            assert rel_err(to_np(got), want) < 2e-2
