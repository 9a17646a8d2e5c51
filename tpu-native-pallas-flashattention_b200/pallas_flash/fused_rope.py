"""FlashAttention with rotary position embeddings applied inside the kernel.

Drop-in for ``src/pallas_flash/fused_rope.py`` of the reference: Q and K are
rotated with ``x*cos + rotate_half(x)*sin`` (fused_rope.py:43-50, :75-78).
On the tensor-core path each query tile is rotated once in shared memory (the
rotated Q never reaches HBM) and each key row is rotated exactly once into a
workspace that the attention kernel streams -- the reference instead rotates
the K block for every (query head, query block) that reads it.  Separate query and
key tables cover decode, where the query sits at position ``pos`` and keys
span ``[0, pos]``.

The reference is forward-only (fused_rope.py:25-27).  Here the function is also
differentiable in q, k and v: when gradients are needed the forward rotates Q
and K with ``pf_rope_apply`` and runs the attention forward that saves the
log-sum-exp; the backward runs the attention backward on the rotated tensors
and maps dQ and dK back through the transposed rotation (sin negated).  The
tables are treated as constants (no gradient).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib
from .flash_attention import _bwd, _fwd

__all__ = ["flash_attention_rope", "rope_apply"]


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, inverse: bool = False,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x*cos + rotate_half(x)*sin`` over ``[B, H, S, D]`` rows on the GPU (fp32 arithmetic).

    ``inverse=True`` applies the transposed rotation (the gradient map).  Row s
    of the ``[S, D]`` tables belongs to position s (fused_rope.py:43-50).
    """
    _lib.require_cuda(x, cos, sin)
    B, H, S, D = x.shape
    if tuple(cos.shape) != (S, D) or tuple(sin.shape) != (S, D):
        raise ValueError(f"cos/sin must have shape {(S, D)}, got {tuple(cos.shape)}, {tuple(sin.shape)}")
    x = x.contiguous()
    cos, sin = cos.contiguous(), sin.to(cos.dtype).contiguous()
    if out is None:
        out = torch.empty_like(x)
    _lib.check(_lib.lib().pf_rope_apply(
        x.data_ptr(), cos.data_ptr(), sin.data_ptr(), _lib.dtype_code(cos.dtype), out.data_ptr(),
        _lib.dtype_code(x.dtype), B, H, S, D, int(bool(inverse)), _lib.stream_of(x)))
    return out


class _RopeAttentionFn(torch.autograd.Function):
    """Differentiable RoPE attention: saves the rotated Q/K, out and lse."""

    @staticmethod
    def forward(ctx, q, k, v, q_cos, q_sin, k_cos, k_sin, causal, sm_scale, kv_len):
        qr = rope_apply(q, q_cos, q_sin)
        kr = rope_apply(k, k_cos, k_sin)
        out, lse = _fwd(qr, kr, v, causal, sm_scale, kv_len, want_lse=True)
        ctx.save_for_backward(qr, kr, v, out, lse, q_cos, q_sin, k_cos, k_sin)
        ctx.causal, ctx.sm_scale, ctx.kv_len = causal, sm_scale, kv_len
        return out

    @staticmethod
    def backward(ctx, do):
        qr, kr, v, out, lse, q_cos, q_sin, k_cos, k_sin = ctx.saved_tensors
        dqr, dkr, dv = _bwd(qr, kr, v, out, lse, do, ctx.causal, ctx.sm_scale, ctx.kv_len)
        dq = rope_apply(dqr, q_cos, q_sin, inverse=True, out=dqr)
        dk = rope_apply(dkr, k_cos, k_sin, inverse=True, out=dkr)
        return dq, dk, dv, None, None, None, None, None, None, None


def flash_attention_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_cos: torch.Tensor,
    q_sin: torch.Tensor,
    k_cos: Optional[torch.Tensor] = None,
    k_sin: Optional[torch.Tensor] = None,
    *,
    causal: bool = False,
    sm_scale: Optional[float] = None,
    block_q: int = 128,
    block_k: int = 128,
    kv_len: Optional[int] = None,
    interpret: bool = False,
) -> torch.Tensor:
    """Attention with RoPE applied to Q and K inside the kernel.

    Numerically ``flash_attention(apply_rope(q), apply_rope(k), v)`` with the
    rotation done in fp32.  Tables are ``[seq_len_q, head_dim]`` and
    ``[seq_len_k, head_dim]``; ``k_cos``/``k_sin`` default to the query
    tables when the two sequence lengths agree (fused_rope.py:154-181 rules).
    """
    del block_q, block_k, interpret
    if k_cos is None or k_sin is None:
        if k.shape[2] != q.shape[2]:
            raise ValueError(
                "k_cos/k_sin are required when the key sequence length differs "
                "from the query sequence length"
            )
        k_cos, k_sin = q_cos, q_sin

    batch, num_heads, seq_len_q, head_dim = q.shape
    num_kv_heads, seq_len_k = k.shape[1], k.shape[2]
    if num_heads % num_kv_heads != 0:
        raise ValueError(
            f"num_heads ({num_heads}) must be a multiple of num_kv_heads ({num_kv_heads})"
        )
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    for name, tbl, want in (("q_cos", q_cos, seq_len_q), ("q_sin", q_sin, seq_len_q),
                            ("k_cos", k_cos, seq_len_k), ("k_sin", k_sin, seq_len_k)):
        if tuple(tbl.shape) != (want, head_dim):
            raise ValueError(f"{name} must have shape {(want, head_dim)}, got {tuple(tbl.shape)}")
    if k.shape != v.shape or k.shape[0] != batch or k.shape[3] != head_dim:
        raise ValueError("k/v must be [batch, num_kv_heads, seq_len_k, head_dim] like q")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    if kv_len is None:
        kv_len = seq_len_k
    elif not 0 < kv_len <= seq_len_k:
        raise ValueError(f"kv_len must be in (0, {seq_len_k}], got {kv_len}")

    _lib.require_cuda(q, k, v, q_cos, q_sin, k_cos, k_sin)
    tdt = q_cos.dtype
    tables = [t.to(tdt).contiguous() for t in (q_cos, q_sin, k_cos, k_sin)]
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError(f"q, k, v must share a dtype, got {q.dtype}, {k.dtype}, {v.dtype}")
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _RopeAttentionFn.apply(q, k, v, *tables, bool(causal), float(sm_scale), int(kv_len))
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty_like(q)
    L = _lib.lib()
    code = _lib.dtype_code(q.dtype)
    ws = _lib.workspace(L.pf_rope_fwd_workspace_size(code, batch, num_kv_heads, seq_len_k, head_dim),
                        q.device)
    _lib.check(L.pf_rope_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), *(t.data_ptr() for t in tables),
        _lib.dtype_code(tdt), out.data_ptr(), code, batch, num_heads,
        num_kv_heads, seq_len_q, seq_len_k, head_dim, int(bool(causal)), float(sm_scale),
        int(kv_len), ws.data_ptr(), ws.numel(), _lib.stream_of(q)))
    return out
