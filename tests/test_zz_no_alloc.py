"""pf_paged_decode_noalloc: paged decode for callers that cannot allocate.

Some callers of this library cannot hand it a scratch buffer -- a host that
manages device memory as fixed arenas, or a call site that only receives its
input and output buffers and may not call cudaMalloc.  For them the library
keeps the split-KV scratch in a fixed 16 MiB array of its own.  These tests
call that entry point through the C ABI and check it against the workspace
entry point (pf_paged_decode, reached through paged_flash_attention) within
the bf16 tolerance the other decode tests use, on two calls in a row (the
scratch keeps the previous call's contents, which must not matter).  The file
name sorts last so a failure here comes after every other test has run.
"""

import ctypes

import numpy as np
import pytest
import torch

import pallas_flash as pf
from pallas_flash import _lib

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _case(B, H, Hkv, ps, D, lens, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    pps = max(lens) // ps + 1
    num_pages = B * pps + 5
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(seed))[: B * pps]
    table = perm.reshape(B, pps).to(torch.int32).cuda()
    kp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    vp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    return q, kp, vp, table, torch.tensor(lens, dtype=torch.int32, device="cuda")


def _noalloc(q, kp, vp, table, lens, max_len):
    B, H, _, D = q.shape
    num_pages, Hkv, ps, _ = kp.shape
    out = torch.empty_like(q)
    st = _lib.lib().pf_paged_decode_noalloc(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), table.data_ptr(), lens.data_ptr(), out.data_ptr(),
        _lib.dtype_code(q.dtype), B, H, Hkv, num_pages, ps, table.shape[1], D, max_len,
        float(1.0 / np.sqrt(D)), torch.cuda.current_stream().cuda_stream)
    return st, out


@pytest.mark.parametrize("B,H,Hkv,ps,D,lens", [
    (4, 8, 2, 16, 128, [1, 100, 1000, 3000]),
    (3, 4, 4, 32, 64, [33, 64, 5]),
    (64, 32, 8, 16, 128, [4096] * 32 + [17] * 32),
])
def test_noalloc_matches_workspace_entry_point_twice(B, H, Hkv, ps, D, lens):
    q, kp, vp, table, ll = _case(B, H, Hkv, ps, D, lens, seed=B + ps)
    max_len = table.shape[1] * ps
    want = pf.paged_flash_attention(q, kp, vp, table, ll, max_context_len=max_len)
    for call in range(2):
        _lib.device_status(reset=True)
        st, got = _noalloc(q, kp, vp, table, ll, max_len)
        assert st == _lib.PF_OK, _lib.lib().pf_last_error().decode()
        torch.cuda.synchronize()
        assert _lib.device_status(reset=True) == 0, call
        err = float((got.float() - want.float()).abs().max())
        assert err < BF16_TOL, (call, err)


def test_noalloc_widened_splits_match_workspace_entry_point():
    """At B=256, H=32, D=128 one split of partials is 4.26 MB, so the 16 MiB scratch
    holds 3 splits where the workspace entry point plans 8: the no-alloc call widens
    the splits to 11008 keys (beyond the 4096-key split that keeps a CTA's page ids
    in shared memory).  Every table entry points into a small shared pool, so the
    memory stays small while some sequences are longer than one widened split."""
    B, H, Hkv, ps, D, pps = 256, 32, 8, 16, 128, 2048
    g = torch.Generator(device="cuda").manual_seed(7)
    num_pages = 97
    kp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    vp = torch.randn((num_pages, Hkv, ps, D), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    table = torch.randint(0, num_pages, (B, pps), generator=torch.Generator().manual_seed(7),
                          dtype=torch.int32).cuda()
    lens = [17 + 13 * i for i in range(B)]
    lens[3], lens[100], lens[200], lens[255] = 11009, 22050, 32768, 30000
    ll = torch.tensor(lens, dtype=torch.int32, device="cuda")
    max_len = pps * ps
    want = pf.paged_flash_attention(q, kp, vp, table, ll, max_context_len=max_len)
    for call in range(2):
        _lib.device_status(reset=True)
        st, got = _noalloc(q, kp, vp, table, ll, max_len)
        assert st == _lib.PF_OK, _lib.lib().pf_last_error().decode()
        torch.cuda.synchronize()
        assert _lib.device_status(reset=True) == 0, call
        err = float((got.float() - want.float()).abs().max())
        assert err < BF16_TOL, (call, err)


def test_noalloc_second_call_with_smaller_batch_ignores_stale_scratch():
    big = _case(8, 8, 2, 16, 128, [2000] * 8, seed=1)
    small = _case(2, 8, 2, 16, 128, [50, 300], seed=2)
    for q, kp, vp, table, ll in (big, small):
        max_len = table.shape[1] * 16
        _lib.device_status(reset=True)
        st, got = _noalloc(q, kp, vp, table, ll, max_len)
        assert st == _lib.PF_OK
        torch.cuda.synchronize()
        assert _lib.device_status(reset=True) == 0
        want = pf.paged_flash_attention(q, kp, vp, table, ll, max_context_len=max_len)
        assert float((got.float() - want.float()).abs().max()) < BF16_TOL


def test_noalloc_rejects_requests_beyond_its_scratch():
    # B*H*(D+2)*4 bytes for one split = 4096*32*130*4 > 16 MiB
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    p = dummy.data_ptr()
    st = _lib.lib().pf_paged_decode_noalloc(p, p, p, p, p, p, 1, 4096, 32, 8, 4, 16, 1, 128, 16, 0.1,
                                            torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PF_ERR_WORKSPACE
    assert "scratch" in _lib.lib().pf_last_error().decode()
