"""Delta preprocess (delta[row] = sum_d o[row, d] * do[row, d], the reference's
flash_attention.py:363-365) called directly through the C ABI, against the
float64 sum of the same (rounded) inputs.  Covers the 16-byte vector kernel for
every dtype and head size, ragged row counts, and the scalar kernel that an
unaligned base pointer or an odd head size selects."""

import numpy as np
import pytest
import torch

from pallas_flash import _lib

pytestmark = pytest.mark.gpu


def _delta(o, do, B, H, S, D):
    out = torch.full((B * H * S,), float("nan"), dtype=torch.float32, device=o.device)
    _lib.check(_lib.lib().pf_bwd_preprocess(o.data_ptr(), do.data_ptr(), out.data_ptr(),
                                            _lib.dtype_code(o.dtype), B, H, S, D,
                                            _lib.stream_of(o)))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 1, 1, 64), (2, 3, 37, 128), (1, 4, 129, 256),
                                   (1, 2, 33, 32), (1, 1, 5, 8), (3, 2, 1000, 128), (1, 1, 7, 72)])
def test_delta_matches_float64(dtype, shape):
    B, H, S, D = shape
    g = torch.Generator().manual_seed(B * 1000 + S)
    o = torch.randn((B, H, S, D), generator=g).to(dtype)
    do = torch.randn((B, H, S, D), generator=g).to(dtype)
    want = (o.double() * do.double()).sum(-1).reshape(-1).numpy()
    got = _delta(o.cuda(), do.cuda(), B, H, S, D)
    tol = 1e-5 * np.abs(o.double()).max().item() * np.abs(do.double()).max().item() * D
    np.testing.assert_allclose(got, want, rtol=0, atol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_delta_unaligned_base_uses_scalar_path(dtype):
    B, H, S, D = 1, 2, 17, 64
    g = torch.Generator().manual_seed(5)
    o = torch.randn((B * H * S * D + 1,), generator=g).to(dtype)
    do = torch.randn((B * H * S * D,), generator=g).to(dtype)
    o_dev = o.cuda()[1:]  # base pointer 2 or 4 bytes past a 16-byte boundary
    want = (o[1:].double() * do.double()).reshape(-1, D).sum(-1).numpy()
    got = _delta(o_dev, do.cuda(), B, H, S, D)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-3)
