"""FlashAttention forward/backward and single-query decode on B200 (sm_100a).

Drop-in for ``src/pallas_flash/flash_attention.py`` of the reference: the same
functions, argument names, defaults, shape rules and ``ValueError`` cases, on
CUDA ``torch.Tensor`` operands instead of ``jax.Array``.  The arithmetic runs
in libpallas_flash_b200.so:

* bf16 / f16 inputs with head_dim 64 or 128 use the tcgen05/TMEM tensor-core
  forward (TMA-fed, fp32 softmax statistics, causal and kv_len tile skipping,
  GQA head mapping in the tile scheduler);
* fp32 inputs (which the reference up-casts and must match to 1e-4
  relative) and other head sizes use fp32 SIMT kernels;
* the backward is the delta preprocess plus dQ and dK/dV kernels, with the
  GQA group-sum done inside the dK/dV kernel.

``flash_attention`` is differentiable through ``torch.autograd`` (the analogue
of the reference's ``jax.custom_vjp``, flash_attention.py:448-476) and saves
``(q, k, v, out, lse)`` as its residuals.  ``block_q``/``block_k`` are accepted
for API compatibility; tile shapes are chosen by the kernels.  ``interpret`` is
accepted and ignored: there is no CPU path.  ``kv_len`` is a runtime value
(no re-compilation per decode position).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

__all__ = ["flash_attention", "flash_attention_decode", "flash_attention_with_lse"]


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_len: Optional[int]) -> int:
    """Shape rules of flash_attention.py:527-545; returns the effective kv_len."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, v must be rank-4 [batch, heads, seq, head_dim] arrays")
    batch, num_heads, _, head_dim = q.shape
    num_kv_heads, seq_len_k = k.shape[1], k.shape[2]
    if k.shape != v.shape:
        raise ValueError("k and v must have the same shape")
    if k.shape[0] != batch or k.shape[3] != head_dim:
        raise ValueError("q and k/v must share batch and head_dim")
    if num_kv_heads == 0 or num_heads % num_kv_heads != 0:
        raise ValueError(
            f"num_heads ({num_heads}) must be a multiple of num_kv_heads "
            f"({num_kv_heads}) for grouped-query attention"
        )
    if kv_len is None:
        return seq_len_k
    kv_len = int(kv_len)
    if not 0 < kv_len <= seq_len_k:
        raise ValueError(f"kv_len must be in (0, {seq_len_k}], got {kv_len}")
    return kv_len


def _same_dtype(q, k, v):
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError(f"q, k, v must share a dtype, got {q.dtype}, {k.dtype}, {v.dtype}")


def _fwd(q, k, v, causal, sm_scale, kv_len, want_lse):
    _lib.require_cuda(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    out = torch.empty_like(q)
    lse = torch.empty((B, H, Sq, 1), dtype=torch.float32, device=q.device) if want_lse else None
    _lib.check(_lib.lib().pf_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _lib.ptr(lse),
        _lib.dtype_code(q.dtype), B, H, Hkv, Sq, Sk, D, int(bool(causal)), float(sm_scale),
        int(kv_len), _lib.stream_of(q)))
    return out, lse


def _bwd(q, k, v, out, lse, do, causal, sm_scale, kv_len):
    q, k, v, out, do = (t.contiguous() for t in (q, k, v, out, do))
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    B, H, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    L = _lib.lib()
    code = _lib.dtype_code(q.dtype)
    ws_bytes = L.pf_bwd_workspace_size(code, B, H, Hkv, Sq, Sk, D, int(bool(causal)), int(kv_len))
    ws = _lib.workspace(ws_bytes, q.device)
    _lib.check(L.pf_bwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), code, B, H, Hkv, Sq, Sk, D,
        int(bool(causal)), float(sm_scale), int(kv_len), ws.data_ptr(), ws.numel(),
        _lib.stream_of(q)))
    return dq, dk, dv


class _FlashAttentionFn(torch.autograd.Function):
    """custom-VJP analogue: forward saves (q, k, v, out, lse)  (flash_attention.py:458-464)."""

    @staticmethod
    def forward(ctx, q, k, v, causal, sm_scale, kv_len):
        out, lse = _fwd(q, k, v, causal, sm_scale, kv_len, want_lse=True)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.sm_scale, ctx.kv_len = causal, sm_scale, kv_len
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = _bwd(q, k, v, out, lse, do, ctx.causal, ctx.sm_scale, ctx.kv_len)
        return dq, dk, dv, None, None, None


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    sm_scale: Optional[float] = None,
    block_q: int = 128,
    block_k: int = 128,
    kv_len: Optional[int] = None,
    interpret: bool = False,
) -> torch.Tensor:
    """FlashAttention on B200: ``softmax(q k^T * sm_scale) v`` without the [Sq, Sk] matrix.

    Args mirror the reference (flash_attention.py:479-526): ``q`` is
    ``[batch, num_heads, seq_len_q, head_dim]``, ``k``/``v`` are
    ``[batch, num_kv_heads, seq_len_k, head_dim]`` with ``num_heads`` a multiple
    of ``num_kv_heads`` (query head ``h`` reads kv head ``h // (H / Hkv)``);
    ``causal`` masks ``k_pos > q_pos`` with both sequences starting at 0;
    ``kv_len`` (default ``seq_len_k``) masks positions ``>= kv_len``;
    ``sm_scale`` defaults to ``1/sqrt(head_dim)``.  Returns an array shaped
    like ``q`` in ``q.dtype``.  Differentiable in q, k, v.
    """
    del block_q, block_k, interpret
    kv_len = _validate(q, k, v, kv_len)
    _same_dtype(q, k, v)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _FlashAttentionFn.apply(q, k, v, bool(causal), float(sm_scale), kv_len)
    out, _ = _fwd(q, k, v, causal, sm_scale, kv_len, want_lse=False)
    return out


def flash_attention_with_lse(q, k, v, *, causal=False, sm_scale=None, kv_len=None):
    """Forward only, returning ``(out, lse)`` with ``lse`` shaped ``[B, H, Sq, 1]`` f32.

    Exposes the residual the reference's forward rule saves
    (flash_attention.py:458-464), for callers that drive the backward themselves.
    """
    kv_len = _validate(q, k, v, kv_len)
    _same_dtype(q, k, v)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    return _fwd(q, k, v, causal, sm_scale, kv_len, want_lse=True)


def flash_attention_backward(q, k, v, out, lse, do, *, causal=False, sm_scale=None, kv_len=None):
    """The VJP of ``flash_attention``: returns ``(dq, dk, dv)`` in the input dtypes.

    Equivalent of ``_flash_attention_bwd_call`` (flash_attention.py:354-442):
    delta preprocess, dQ, and dK/dV already summed over each GQA group.
    """
    kv_len = _validate(q, k, v, kv_len)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    _lib.require_cuda(q, k, v, out, lse, do)
    return _bwd(q, k, v, out, lse.contiguous(), do, causal, sm_scale, kv_len)


def flash_attention_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cache_len: int,
    *,
    sm_scale: Optional[float] = None,
    block_k: int = 128,
    interpret: bool = False,
) -> torch.Tensor:
    """Single-token decode against a fixed-size KV cache (flash_attention.py:555-589).

    ``q`` is ``[batch, num_heads, 1, head_dim]``; the caches are
    ``[batch, num_kv_heads, cache_size, head_dim]``; positions
    ``[0, cache_len)`` are attended and nothing past ``cache_len`` is read.
    ``cache_len`` is a runtime scalar.  Runs the split-KV decode kernel, which
    reads each cached K/V row once for the whole query-head group.
    """
    del block_k, interpret
    if q.shape[2] != 1:
        raise ValueError(f"decode expects a single query row, got seq_len_q={q.shape[2]}")
    cache_len = _validate(q, k_cache, v_cache, cache_len)
    _same_dtype(q, k_cache, v_cache)
    _lib.require_cuda(q, k_cache, v_cache)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    q, k_cache, v_cache = q.contiguous(), k_cache.contiguous(), v_cache.contiguous()
    B, H, _, D = q.shape
    Hkv, C = k_cache.shape[1], k_cache.shape[2]
    out = torch.empty_like(q)
    L = _lib.lib()
    ws = _lib.workspace(L.pf_decode_workspace_size(B, H, Hkv, C, D), q.device)
    _lib.check(L.pf_decode(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
        _lib.dtype_code(q.dtype), B, H, Hkv, C, D, int(cache_len), float(sm_scale),
        ws.data_ptr(), ws.numel(), _lib.stream_of(q)))
    return out
