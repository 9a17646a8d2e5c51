"""ctypes binding of libpallas_flash_b200.so (the C ABI in include/pallas_flash_b200.h).

This is the only way the Python API reaches the GPU: there is no CPU, XLA or
PyTorch fallback.  If the shared library is missing the first call raises
``RuntimeError`` (build it with ``python tpu-native-pallas-flashattention_b200/build.py``).
PyTorch supplies device memory, the current CUDA stream and the caching
allocator for workspaces; the kernels are the library's own.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpallas_flash_b200.so"

PF_OK = 0
PF_ERR_INVALID = 1
PF_ERR_UNSUPPORTED = 2
PF_ERR_CUDA = 3
PF_ERR_DEVICE = 4
PF_ERR_WORKSPACE = 5

PF_DEV_WAIT_TIMEOUT = 1
PF_DEV_BAD_PAGE = 2
PF_DEV_SMEM_LAYOUT = 4
PF_DEV_LEN_OVER_MAX = 8

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_L = ctypes.c_long

# name -> (restype, argtypes); mirrors include/pallas_flash_b200.h
_SIGNATURES = {
    "pf_last_error": (ctypes.c_char_p, []),
    "pf_version": (ctypes.c_char_p, []),
    "pf_device_status": (_I, [ctypes.POINTER(_I), _I]),
    "pf_set_wait_limit_ns": (_I, [ctypes.c_ulonglong]),
    "pf_selftest_wait_timeout": (_I, [_P]),
    "pf_fwd_kernel_kind": (_I, [_I, _I]),
    "pf_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "pf_rope_fwd_workspace_size": (_Z, [_I, _I, _I, _I, _I]),
    "pf_rope_fwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _Z, _P]),
    "pf_add_rms_norm": (_I, [_P, _P, _P, _P, _P, _I, _L, _I, _F, _P]),
    "pf_silu_mul": (_I, [_P, _P, _P, _I, _L, _I, _L, _P]),
    "pf_rows_linear": (_I, [_P, _P, _F, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "pf_rows_linear_rope_write": (_I, [_P, _P, _F, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I,
                                       _I, _I, _I, _I, _P]),
    "pf_decode_positions": (_I, [_P, _I, _P, _P, _P, _I, _P]),
    "pf_argmax_embed": (_I, [_P, _L, _I, _I, _P, _P, _P, _I, _I, _P]),
    "pf_bwd_preprocess": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "pf_bwd_head_parts": (_I, [_I, _I, _I, _I]),
    "pf_bwd_dq": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "pf_bwd_dkv": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "pf_bwd_workspace_size": (_Z, [_I, _I, _I, _I, _I, _I, _I, _I, _I]),
    "pf_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _Z, _P]),
    "pf_decode_workspace_size": (_Z, [_I, _I, _I, _I, _I]),
    "pf_decode": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P]),
    "pf_paged_decode_workspace_size": (_Z, [_I, _I, _I, _I, _I, _I]),
    "pf_paged_decode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P]),
    "pf_paged_decode_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P]),
    "pf_paged_write": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "pf_cache_write": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "pf_paged_gather": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "pf_paged_prefill_workspace_size": (_Z, [_I, _I, _I, _I, _I]),
    "pf_paged_prefill": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P]),
    "pf_rope_apply": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _P]),
    "pf_rope_paged_write": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                 _P]),
    "pf_rope_paged_write_qkv": (_I, [_P, _L, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                     _I, _P]),
}

EXPORTED = tuple(_SIGNATURES)


def load_library(path: Path | str | None = None) -> ctypes.CDLL:
    """Loads (once) and returns the shared library with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"pallas_flash native library not found at {p}; build it with "
                "`python tpu-native-pallas-flashattention_b200/build.py` (no CPU fallback exists)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load_library()


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPES[t]
    except KeyError:
        raise ValueError(f"unsupported dtype {t}; expected float32, bfloat16 or float16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(
                "pallas_flash runs only on CUDA tensors (sm_100a kernels; there is no CPU or "
                "interpret-mode fallback)"
            )


def check(status: int) -> None:
    """Maps a C-ABI status to the reference's exception types."""
    if status == PF_OK:
        return
    msg = lib().pf_last_error().decode(errors="replace")
    if status == PF_ERR_INVALID:
        raise ValueError(msg)
    if status == PF_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"pallas_flash error {status}: {msg}")


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def device_status(reset: bool = True) -> int:
    """Device status bits recorded by the kernels (synchronises the device)."""
    v = ctypes.c_int(0)
    check(lib().pf_device_status(ctypes.byref(v), 1 if reset else 0))
    return v.value


def forward_kernel_kind(dtype: torch.dtype, head_dim: int) -> str:
    return "tcgen05" if lib().pf_fwd_kernel_kind(dtype_code(dtype), head_dim) == 1 else "simt"
