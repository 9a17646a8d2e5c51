"""Paged decode on the GPU (port of the reference's tests/test_paged.py) plus
bit-exact block-table indexing checks."""

import numpy as np
import pytest
import torch

import pallas_flash as pf
from pallas_flash import _lib
from oracle import attention_oracle as orc
from conftest import randn, to_dev, to_np, widen

pytestmark = pytest.mark.gpu


def scrambled_table(batch, pages_per_seq, num_pages, seed):
    rng = np.random.default_rng(seed)
    return np.stack([rng.choice(num_pages, size=pages_per_seq, replace=False) for _ in range(batch)]).astype(np.int32)


@pytest.mark.parametrize("batch,n_heads,n_kv_heads,page_size,context_lens", [
    (1, 2, 2, 64, [100]),
    (3, 4, 2, 64, [10, 130, 200]),
    (2, 4, 1, 128, [128, 5]),
    (4, 2, 2, 32, [1, 33, 64, 90]),
    (5, 8, 2, 16, [1, 16, 17, 300, 511]),
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_paged_matches_contiguous(batch, n_heads, n_kv_heads, page_size, context_lens, dtype):
    dim = 128
    pages_per_seq = max(context_lens) // page_size + 1
    num_pages = max(32, batch * pages_per_seq)
    q = randn((batch, n_heads, 1, dim), 0)
    kp, vp = randn((num_pages, n_kv_heads, page_size, dim), 1), randn((num_pages, n_kv_heads, page_size, dim), 2)
    table = scrambled_table(batch, pages_per_seq, num_pages, seed=batch)
    tq, tkp, tvp = (to_dev(x, dtype) for x in (q, kp, vp))
    out = pf.paged_flash_attention(tq, tkp, tvp, to_dev(table), torch.tensor(context_lens, dtype=torch.int32))
    assert out.shape == q.shape
    ref = orc.paged_attention(widen(tq), widen(tkp), widen(tvp), table, np.array(context_lens))
    tol = 2e-3 if dtype == torch.float32 else 2e-2
    assert np.max(np.abs(to_np(out) - ref)) < tol


def test_pages_are_shareable():
    dim, page_size, num_pages = 128, 64, 8
    q1 = randn((1, 2, 1, dim), 7)
    q = np.concatenate([q1, q1])
    kp, vp = randn((num_pages, 2, page_size, dim), 8), randn((num_pages, 2, page_size, dim), 9)
    out = pf.paged_flash_attention(to_dev(q), to_dev(kp), to_dev(vp),
                                   torch.tensor([[3, 5], [3, 5]], dtype=torch.int32),
                                   torch.tensor([100, 100], dtype=torch.int32))
    assert torch.equal(out[0], out[1])


def test_unwritten_pages_do_not_leak():
    page_size, dim = 64, 128
    kp = torch.cat([torch.ones((1, 2, page_size, dim)), torch.full((1, 2, page_size, dim), float("nan"))]).cuda()
    q = torch.ones((1, 2, 1, dim), device="cuda")
    out = pf.paged_flash_attention(q, kp, kp, torch.tensor([[0, 1]], dtype=torch.int32),
                                   torch.tensor([page_size], dtype=torch.int32))
    assert torch.isfinite(out).all()
    assert torch.allclose(out, torch.ones_like(out), atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_trailing_table_entries_never_read(dtype):
    """Entries past the context may be garbage (even out of range): never dereferenced."""
    kp, vp = randn((4, 2, 16, 64), 1), randn((4, 2, 16, 64), 2)
    q = randn((1, 4, 1, 64), 3)
    table = np.array([[2, 0, 10**6, -5]], dtype=np.int32)
    _lib.device_status(reset=True)
    tq, tkp, tvp = (to_dev(x, dtype) for x in (q, kp, vp))
    out = pf.paged_flash_attention(tq, tkp, tvp, to_dev(table), torch.tensor([20], dtype=torch.int32))
    kc = orc.gather_contiguous(widen(tkp), [2, 0], 2, 20)[None]
    vc = orc.gather_contiguous(widen(tvp), [2, 0], 2, 20)[None]
    ref = orc.reference_attention(widen(tq), kc, vc)
    assert np.max(np.abs(to_np(out) - ref)) < (2e-3 if dtype == torch.float32 else 2e-2)
    assert _lib.device_status(reset=True) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_bad_page_id_is_flagged_not_faulted(dtype):
    kp, vp = randn((4, 2, 16, 64), 1), randn((4, 2, 16, 64), 2)
    q = randn((1, 4, 1, 64), 3)
    _lib.device_status(reset=True)
    pf.paged_flash_attention(to_dev(q, dtype), to_dev(kp, dtype), to_dev(vp, dtype),
                             torch.tensor([[1, 99]], dtype=torch.int32), torch.tensor([20], dtype=torch.int32))
    assert _lib.device_status(reset=True) & _lib.PF_DEV_BAD_PAGE


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_length_above_max_context_len_is_flagged_or_rejected(dtype):
    """A length beyond max_context_len is never silently truncated: device lengths
    raise PF_DEV_LEN_OVER_MAX in the status word, host lengths raise ValueError."""
    kp, vp = randn((64, 2, 16, 128), 4), randn((64, 2, 16, 128), 5)
    q = randn((2, 4, 1, 128), 6)
    table = torch.arange(64, dtype=torch.int32).reshape(2, 32)
    args = (to_dev(q, dtype), to_dev(kp, dtype), to_dev(vp, dtype), table.cuda())
    _lib.device_status(reset=True)
    pf.paged_flash_attention(*args, torch.tensor([100, 300], dtype=torch.int32, device="cuda"),
                             max_context_len=300)
    assert _lib.device_status(reset=True) == 0
    pf.paged_flash_attention(*args, torch.tensor([100, 500], dtype=torch.int32, device="cuda"),
                             max_context_len=300)
    assert _lib.device_status(reset=True) & _lib.PF_DEV_LEN_OVER_MAX
    with pytest.raises(ValueError):
        pf.paged_flash_attention(*args, torch.tensor([100, 500], dtype=torch.int32), max_context_len=300)


@pytest.mark.parametrize("page_size", [8, 12, 48, 256])
@pytest.mark.parametrize("D", [64, 128])
def test_page_sizes_bf16(page_size, D):
    """Page sizes on and off the tensor-core path (8/16/32k use TMA segments; others bulk copies)."""
    B, H, Hkv = 3, 8, 2
    lens = [1, page_size * 3 + 5, 700]
    pps = max(lens) // page_size + 1
    num_pages = B * pps + 3
    q = randn((B, H, 1, D), 31)
    kp, vp = randn((num_pages, Hkv, page_size, D), 32), randn((num_pages, Hkv, page_size, D), 33)
    table = scrambled_table(B, pps, num_pages, 4)
    tq, tkp, tvp = (to_dev(x, torch.bfloat16) for x in (q, kp, vp))
    out = pf.paged_flash_attention(tq, tkp, tvp, to_dev(table), torch.tensor(lens, dtype=torch.int32))
    ref = orc.paged_attention(widen(tq), widen(tkp), widen(tvp), table, np.array(lens))
    assert np.max(np.abs(to_np(out) - ref)) < 2e-2


def test_nan_inside_last_partial_page_bf16():
    """NaN in rows past the context inside a page that is read must not leak (rows zeroed)."""
    ps, D = 16, 128
    kp = torch.ones((3, 2, ps, D))
    kp[1, :, 5:] = float("nan")
    kp = kp.to(torch.bfloat16).cuda()
    q = torch.ones((1, 4, 1, D), dtype=torch.bfloat16, device="cuda")
    out = pf.paged_flash_attention(q, kp, kp, torch.tensor([[0, 1, 2]], dtype=torch.int32),
                                   torch.tensor([ps + 5], dtype=torch.int32))
    assert torch.isfinite(out.float()).all()
    assert torch.allclose(out.float(), torch.ones_like(out, dtype=torch.float32), atol=1e-5)


def test_write_to_paged_cache_roundtrip():
    page_size, dim, n_kv, num_pages, length = 32, 128, 2, 4, 70
    k_pages, v_pages = pf.init_paged_cache(num_pages, n_kv, page_size, dim)
    table = torch.tensor([0, 2, 1, 3], dtype=torch.int32)
    ks, vs = randn((1, n_kv, length, dim), 11), randn((1, n_kv, length, dim), 12)
    tks, tvs = to_dev(ks), to_dev(vs)
    for pos in range(length):
        k_pages, v_pages = pf.write_to_paged_cache(k_pages, v_pages, tks[:, :, pos:pos + 1],
                                                   tvs[:, :, pos:pos + 1], table, pos)
    q = randn((1, 2, 1, dim), 13)
    out = pf.paged_flash_attention(to_dev(q), k_pages, v_pages, table[None], torch.tensor([length], dtype=torch.int32))
    assert np.max(np.abs(to_np(out) - orc.reference_attention(q, ks, vs))) < 2e-3
    # byte-exact placement against the oracle's writer
    okp = np.zeros((num_pages, n_kv, page_size, dim), np.float32)
    ovp = np.zeros_like(okp)
    for pos in range(length):
        orc.paged_write(okp, ovp, ks[:, :, pos:pos + 1], vs[:, :, pos:pos + 1], table.numpy(), pos)
    assert np.array_equal(k_pages.cpu().numpy(), okp) and np.array_equal(v_pages.cpu().numpy(), ovp)


def test_write_out_of_table_raises_index_error():
    k_pages, v_pages = pf.init_paged_cache(4, 2, 32, 128)
    x = torch.zeros((1, 2, 1, 128), device="cuda")
    with pytest.raises(IndexError):
        pf.write_to_paged_cache(k_pages, v_pages, x, x, torch.tensor([0, 1], dtype=torch.int32), 64)


def test_gather_is_byte_exact():
    pool = torch.randn((64, 4, 16, 128), device="cuda").to(torch.bfloat16)
    table = scrambled_table(5, 12, 64, 3)
    got = pf.gather_paged(pool, to_dev(table))
    want = np.stack([orc.gather_contiguous(pool.view(torch.int16).cpu().numpy(), table[b], 12, 12 * 16)
                     for b in range(5)])
    assert np.array_equal(got.view(torch.int16).cpu().numpy(), want)


def test_paged_equals_fixed_cache_bitwise():
    """Same split schedule => paged decode over a scrambled pool == fixed-cache decode of the gather."""
    B, H, Hkv, ps, D, pps = 4, 8, 2, 16, 128, 64
    cap = ps * pps
    num_pages = B * pps + 7
    g = torch.Generator(device="cuda").manual_seed(5)
    pool_k = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    pool_v = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    table = to_dev(scrambled_table(B, pps, num_pages, 9))
    kc, vc = pf.gather_paged(pool_k, table), pf.gather_paged(pool_v, table)
    for L in (cap, 700, 33):
        paged = pf.paged_flash_attention(q, pool_k, pool_v, table, torch.full((B,), L, dtype=torch.int32),
                                         max_context_len=cap)
        fixed = pf.flash_attention_decode(q, kc, vc, L)
        assert torch.equal(paged, fixed), L


def test_c4_shape_sampled():
    """BASELINE config 4 shape (page 16, H32/Hkv8/D128) on 16 sequences, ragged lengths."""
    rng = np.random.default_rng(0)
    B, H, Hkv, ps, D = 16, 32, 8, 16, 128
    lens = rng.integers(512, 32769, size=B)
    pages = [(int(L) + ps - 1) // ps for L in lens]
    pool = int(np.ceil(1.1 * sum(pages)))
    perm = rng.permutation(pool)
    pps = max(pages)
    table = np.zeros((B, pps), np.int32)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    g = torch.Generator(device="cuda").manual_seed(1)
    kp = torch.randn((pool, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    vp = torch.randn((pool, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    out = pf.paged_flash_attention(q, kp, vp, to_dev(table), torch.tensor(lens, dtype=torch.int32))
    for b in (0, 7, 15):
        kc = pf.gather_paged(kp, to_dev(table[b:b + 1]))[:, :, :lens[b]]
        vc = pf.gather_paged(vp, to_dev(table[b:b + 1]))[:, :, :lens[b]]
        ref = orc.reference_attention(widen(q[b:b + 1]), widen(kc), widen(vc), dtype=np.float32)
        assert np.max(np.abs(to_np(out[b:b + 1]) - ref)) < 2e-2


def test_sequence_sharding_is_bitwise_identical():
    """Each rank's local pool + remapped table gives the same bits as the full problem."""
    from pallas_flash import sharding
    rng = np.random.default_rng(2)
    B, H, Hkv, ps, D = 12, 8, 2, 16, 128
    lens = rng.integers(1, 2000, size=B)
    pps = int(lens.max()) // ps + 1
    num_pages = B * pps
    table = scrambled_table(B, pps, num_pages, 5)
    g = torch.Generator(device="cuda").manual_seed(6)
    kp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    vp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    tt, ll = to_dev(table), torch.tensor(lens, dtype=torch.int32, device="cuda")
    cap = pps * ps
    full = pf.paged_flash_attention(q, kp, vp, tt, ll, max_context_len=cap)
    for seqs in sharding.greedy_balance(lens, 3):
        ql, kl, vl, tl, lt = sharding.local_paged_problem(q, kp, vp, tt, ll, seqs)
        tl = torch.nn.functional.pad(tl, (0, pps - tl.shape[1]))
        part = pf.paged_flash_attention(ql, kl, vl, tl, lt, max_context_len=cap)
        assert torch.equal(part, full[seqs]), seqs


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,D,ps", [(8, 2, 64, 16), (4, 4, 128, 8)])
def test_rope_paged_write_matches_unfused(dtype, H, Hkv, D, ps):
    """Fused decode prologue == apply_rope on q/k (fp32, one rounding) + the page write."""
    B, pps, rows = 5, 6, 100
    num_pages = B * pps + 3
    rng = np.random.default_rng(7)
    q = randn((B, H, 1, D), 1)
    k = randn((B, Hkv, 1, D), 2)
    v = randn((B, Hkv, 1, D), 3)
    cos, sin = pf.precompute_rope(rows, D, 10000.0, device="cuda")
    tables = rng.permutation(num_pages)[: B * pps].reshape(B, pps).astype(np.int32)
    positions = rng.integers(0, pps * ps, size=B).astype(np.int32)
    rope_rows = rng.integers(0, rows, size=B).astype(np.int32)
    kp0 = randn((num_pages, Hkv, ps, D), 4)
    vp0 = randn((num_pages, Hkv, ps, D), 5)
    tq = to_dev(q, dtype)
    kp, vp = to_dev(kp0, dtype), to_dev(vp0, dtype)
    out = pf.rope_write_to_paged_cache_batch(tq, to_dev(k, dtype), to_dev(v, dtype), kp, vp, cos, sin,
                                             torch.from_numpy(tables), torch.from_numpy(positions),
                                             torch.from_numpy(rope_rows))
    assert out.data_ptr() == tq.data_ptr()  # rotated in place
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    qw, kw, vw = widen(to_dev(q, dtype)), widen(to_dev(k, dtype)), widen(to_dev(v, dtype))
    kp_want, vp_want = widen(to_dev(kp0, dtype)), widen(to_dev(vp0, dtype))
    for b in range(B):
        r = rope_rows[b]
        want_q = orc.apply_rope(qw[b:b + 1], c[r:r + 1], s[r:r + 1])
        assert np.max(np.abs(to_np(tq[b:b + 1]) - want_q)) <= tol * max(1.0, np.max(np.abs(want_q)))
        page, off = tables[b, positions[b] // ps], positions[b] % ps
        kp_want[page, :, off] = orc.apply_rope(kw[b:b + 1], c[r:r + 1], s[r:r + 1])[0, :, 0]
        vp_want[page, :, off] = vw[b, :, 0]
    np.testing.assert_allclose(widen(kp), kp_want, rtol=0, atol=tol * 8)
    assert np.array_equal(widen(vp), vp_want)  # v and every untouched slot byte-exact


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,D,ps", [(8, 2, 64, 16), (4, 4, 128, 8)])
def test_rope_paged_write_qkv_equals_separate_tensors(dtype, H, Hkv, D, ps):
    """One fused projection row per sequence (q heads, k heads, v heads) gives
    byte-identical q and pages to the separate-tensor entry point."""
    B, pps, rows = 5, 6, 100
    num_pages = B * pps + 3
    rng = np.random.default_rng(8)
    qkv = to_dev(randn((B, 1, (H + 2 * Hkv) * D), 11), dtype)
    q = qkv[..., :H * D].reshape(B, 1, H, D).transpose(1, 2).contiguous()
    k = qkv[..., H * D:(H + Hkv) * D].reshape(B, 1, Hkv, D).transpose(1, 2).contiguous()
    v = qkv[..., (H + Hkv) * D:].reshape(B, 1, Hkv, D).transpose(1, 2).contiguous()
    cos, sin = pf.precompute_rope(rows, D, 10000.0, device="cuda")
    tables = torch.from_numpy(rng.permutation(num_pages)[: B * pps].reshape(B, pps).astype(np.int32))
    positions = torch.from_numpy(rng.integers(0, pps * ps, size=B).astype(np.int32))
    rope_rows = torch.from_numpy(rng.integers(0, rows, size=B).astype(np.int32))
    kp0, vp0 = to_dev(randn((num_pages, Hkv, ps, D), 12), dtype), to_dev(randn((num_pages, Hkv, ps, D), 13), dtype)
    kp1, vp1, kp2, vp2 = kp0.clone(), vp0.clone(), kp0.clone(), vp0.clone()
    want = pf.rope_write_to_paged_cache_batch(q, k, v, kp1, vp1, cos, sin, tables, positions, rope_rows)
    got = pf.rope_write_to_paged_cache_qkv(qkv, H, kp2, vp2, cos, sin, tables, positions, rope_rows)
    assert got.shape == (B, H, 1, D) and got.is_contiguous()
    assert torch.equal(got, want)
    assert torch.equal(kp2, kp1) and torch.equal(vp2, vp1)


# --------------------------------------------------------------------------
# Paged (chunked) prefill -- an extension: the reference pages single-query
# decode only.  Oracle: the chunk's L queries are the last rows of a causal
# attention over the gathered context, i.e. reference_attention of a
# full-length query whose last L rows are the chunk, restricted to those rows.
def _prefill_oracle(q, k_pages, v_pages, tables, lens):
    B, H, L, D = q.shape
    pps = tables.shape[1]
    out = np.zeros(q.shape)
    for b, ctx in enumerate(lens):
        kc = orc.gather_contiguous(k_pages, tables[b], pps, ctx)[None]
        vc = orc.gather_contiguous(v_pages, tables[b], pps, ctx)[None]
        q_full = np.zeros((1, H, ctx, D))
        q_full[:, :, ctx - L:] = q[b:b + 1]
        out[b] = orc.reference_attention(q_full, kc, vc, causal=True, dtype=np.float64)[0, :, ctx - L:]
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,D,ps,lens,L", [
    (4, 2, 128, 16, [300, 130, 77], 64),
    (8, 2, 64, 32, [40, 512], 40),
    (4, 4, 128, 16, [1000, 129], 129),
    (2, 1, 128, 8, [257], 256),
    (4, 2, 128, 128, [300, 1000, 77], 64),
    (8, 2, 64, 256, [40, 700], 40),
])
def test_paged_prefill_matches_oracle(dtype, H, Hkv, D, ps, lens, L):
    B = len(lens)
    pps = max((n + ps - 1) // ps for n in lens) + 1
    num_pages = B * pps + 5
    tables = scrambled_table(B, pps, num_pages, seed=3)
    q = randn((B, H, L, D), 41)
    k_pages = randn((num_pages, Hkv, ps, D), 42)
    v_pages = randn((num_pages, Hkv, ps, D), 43)
    tq, tk, tv = to_dev(q, dtype), to_dev(k_pages, dtype), to_dev(v_pages, dtype)
    got = pf.paged_prefill_attention(tq, tk, tv, torch.from_numpy(tables), torch.tensor(lens, dtype=torch.int32))
    assert got.shape == q.shape and got.dtype == dtype
    want = _prefill_oracle(widen(tq), widen(tk), widen(tv), tables, lens)
    tol = 2e-3 if dtype == torch.float32 else 2e-2
    assert np.max(np.abs(to_np(got) - want)) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_paged_prefill_reads_no_ungathered_workspace_row(dtype):
    """The gather writes only rows below each context's next 128-row boundary; the
    workspace is NaN-poisoned first, so a prefill kernel reading any row past that
    would put NaN in the output.  Very unequal contexts leave most rows unwritten."""
    from pallas_flash import _lib
    H, Hkv, D, ps, L = 4, 2, 128, 16, 32
    lens = [1500, 33, 200, 129]
    B = len(lens)
    pps = max((n + ps - 1) // ps for n in lens) + 1
    num_pages = B * pps + 5
    tables = scrambled_table(B, pps, num_pages, seed=9)
    q, kp, vp = randn((B, H, L, D), 51), randn((num_pages, Hkv, ps, D), 52), randn((num_pages, Hkv, ps, D), 53)
    tq, tk, tv = to_dev(q, dtype), to_dev(kp, dtype), to_dev(vp, dtype)
    lib, code = _lib.lib(), _lib.dtype_code(dtype)
    cap = pps * ps
    ws = torch.empty(lib.pf_paged_prefill_workspace_size(code, B, Hkv, cap, D), dtype=torch.uint8, device="cuda")
    ws.view(torch.int32).fill_(-1)  # all-ones bit patterns: NaN in f32 and bf16 alike
    ttab = torch.from_numpy(tables).cuda()
    tlen = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty_like(tq)
    _lib.check(lib.pf_paged_prefill(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), ttab.data_ptr(), tlen.data_ptr(),
                                    out.data_ptr(), code, B, H, Hkv, L, num_pages, ps, pps, D, cap,
                                    1.0 / np.sqrt(D), ws.data_ptr(), ws.numel(), _lib.stream_of(tq)))
    got = to_np(out)
    assert np.isfinite(got).all()
    want = _prefill_oracle(widen(tq), widen(tk), widen(tv), tables, lens)
    tol = 2e-3 if dtype == torch.float32 else 2e-2
    assert np.max(np.abs(got - want)) < tol


@pytest.mark.parametrize("ps", [8, 16, 128])
def test_paged_prefill_ignores_pool_rows_past_the_context(ps):
    """Rows at or past a sequence's length (the rest of its last page, pages it does
    not own) are NaN-poisoned, so reading or multiplying any of them shows up as NaN:
    the context gather must copy only live rows and zero-fill the rest of the tile."""
    dtype = torch.bfloat16
    H, Hkv, D, L = 4, 2, 128, 48
    lens = [700, 49, 130, 256]
    B = len(lens)
    pps = max((n + ps - 1) // ps for n in lens) + 2
    num_pages = B * pps + 5
    tables = scrambled_table(B, pps, num_pages, seed=17)
    q, kp, vp = randn((B, H, L, D), 61), randn((num_pages, Hkv, ps, D), 62), randn((num_pages, Hkv, ps, D), 63)
    live = np.zeros((num_pages, ps), dtype=bool)
    for b, n in enumerate(lens):
        for t in range(n):
            live[tables[b, t // ps], t % ps] = True
    kp = np.where(live[:, None, :, None], kp, np.nan)
    vp = np.where(live[:, None, :, None], vp, np.nan)
    tq, tk, tv = to_dev(q, dtype), to_dev(kp, dtype), to_dev(vp, dtype)
    got = pf.paged_prefill_attention(tq, tk, tv, torch.from_numpy(tables), torch.tensor(lens, dtype=torch.int32))
    out = to_np(got)
    assert np.isfinite(out).all()
    want = _prefill_oracle(widen(tq), widen(tk), widen(tv), tables, lens)
    assert np.max(np.abs(out - want)) < 2e-2


def test_paged_prefill_single_token_equals_paged_decode():
    """L = 1 is the decode case: same math as paged_flash_attention (different kernels)."""
    B, H, Hkv, D, ps = 3, 8, 2, 128, 16
    lens = [100, 17, 260]
    pps = 20
    num_pages = B * pps + 1
    tables = torch.from_numpy(scrambled_table(B, pps, num_pages, seed=5))
    q = to_dev(randn((B, H, 1, D), 51), torch.bfloat16)
    kp = to_dev(randn((num_pages, Hkv, ps, D), 52), torch.bfloat16)
    vp = to_dev(randn((num_pages, Hkv, ps, D), 53), torch.bfloat16)
    ctx = torch.tensor(lens, dtype=torch.int32)
    a = pf.paged_prefill_attention(q, kp, vp, tables, ctx)
    b = pf.paged_flash_attention(q, kp, vp, tables, ctx)
    assert float((a.float() - b.float()).abs().max()) < 2e-2


def test_bounded_wait_times_out_with_a_status_not_a_hang():
    """A wait on an mbarrier nothing arrives on gives up after the (test-shortened)
    limit, records PF_DEV_WAIT_TIMEOUT and the kernel returns; the context stays
    usable for the next call."""
    L = _lib.lib()
    _lib.device_status(reset=True)
    assert L.pf_set_wait_limit_ns(2_000_000) == _lib.PF_OK  # 2 ms
    try:
        assert L.pf_selftest_wait_timeout(torch.cuda.current_stream().cuda_stream) == _lib.PF_OK
        torch.cuda.synchronize()
        assert _lib.device_status(reset=True) & _lib.PF_DEV_WAIT_TIMEOUT
    finally:
        assert L.pf_set_wait_limit_ns(0) == _lib.PF_OK
    # the device still works, and ordinary calls raise no flag
    kp, vp = randn((4, 2, 16, 64), 1), randn((4, 2, 16, 64), 2)
    out = pf.paged_flash_attention(to_dev(randn((1, 4, 1, 64), 3), torch.bfloat16), to_dev(kp, torch.bfloat16),
                                   to_dev(vp, torch.bfloat16), torch.tensor([[1, 2]], dtype=torch.int32),
                                   torch.tensor([20], dtype=torch.int32))
    assert torch.isfinite(out.float()).all()
    assert _lib.device_status(reset=True) == 0
