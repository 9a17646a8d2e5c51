"""The C-ABI library: it loads, exports exactly what include/*.h declares, and
rejects invalid arguments the way the reference raises ValueError -- all
without a GPU (validation precedes any CUDA call)."""

import ctypes
import re
from pathlib import Path

import pytest

from pallas_flash import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "pallas_flash_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pf_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    lib = _lib.load_library()
    assert lib.pf_version().decode().startswith("0.1.0")


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in {HEADER.name} but not exported"


def test_python_binding_covers_header():
    assert sorted(_lib.EXPORTED) == declared_symbols()


def _fwd(H=4, Hkv=4, kv_len=8, dtype=1, D=64):
    lib = _lib.load_library()
    dummy = 256
    return lib.pf_fwd(dummy, dummy, dummy, dummy, None, dtype, 1, H, Hkv, 8, 8, D, 0, 0.1, kv_len, None)


def test_rejects_non_divisible_heads():
    assert _fwd(H=6, Hkv=4) == _lib.PF_ERR_INVALID
    assert "multiple of num_kv_heads" in _lib.lib().pf_last_error().decode()


@pytest.mark.parametrize("kv_len", [0, 9, -1])
def test_rejects_kv_len_out_of_range(kv_len):
    assert _fwd(kv_len=kv_len) == _lib.PF_ERR_INVALID
    assert "kv_len must be in (0, 8]" in _lib.lib().pf_last_error().decode()


def test_rejects_bad_dtype_and_big_head_dim():
    assert _fwd(dtype=7) == _lib.PF_ERR_INVALID
    assert _fwd(D=512) == _lib.PF_ERR_UNSUPPORTED


def test_rope_rejects_odd_head_dim():
    lib = _lib.load_library()
    st = lib.pf_rope_fwd(256, 256, 256, 256, 256, 256, 256, 0, 256, 0, 1, 2, 2, 4, 4, 5, 0, 0.1, 4, None, 0, None)
    assert st == _lib.PF_ERR_INVALID
    assert "even" in lib.pf_last_error().decode()


def test_workspace_queries_and_missing_workspace():
    lib = _lib.load_library()
    n = lib.pf_decode_workspace_size(256, 32, 8, 32768, 128)
    # 8 splits of 4096 keys: [B, H, splits, D + 2] f32
    assert n == 256 * 32 * 8 * 130 * 4
    assert lib.pf_paged_decode_workspace_size(256, 32, 8, 16, 32768, 128) == n
    st = lib.pf_decode(256, 256, 256, 256, 1, 1, 2, 2, 64, 128, 10, 0.1, None, 0, None)
    assert st == _lib.PF_ERR_WORKSPACE
    # delta + the causal dS spill: 528 of the 32 x 32 tile pairs per plane, 32 KiB each
    assert lib.pf_bwd_workspace_size(1, 4, 32, 8, 4096, 4096, 128, 1, 4096) == \
        4 * 32 * 4096 * 4 + 4 * 32 * 528 * 32768
    assert lib.pf_bwd_workspace_size(1, 4, 32, 8, 4096, 4096, 128, 0, 0) == \
        4 * 32 * 4096 * 4 + 4 * 32 * 1024 * 32768
    assert lib.pf_bwd_workspace_size(0, 4, 32, 8, 4096, 4096, 128, 1, 4096) == 4 * 32 * 4096 * 4  # fp32: no spill


def test_paged_decode_validation():
    lib = _lib.load_library()
    st = lib.pf_paged_decode(256, 256, 256, 256, 256, 256, 1, 2, 6, 4, 8, 16, 4, 128, 64, 0.1, 256, 1 << 20, None)
    assert st == _lib.PF_ERR_INVALID
    st = lib.pf_paged_decode(256, 256, 256, 256, 256, 256, 1, 2, 4, 4, 8, 16, 4, 96, 64, 0.1, 256, 1 << 20, None)
    assert st == _lib.PF_ERR_UNSUPPORTED
