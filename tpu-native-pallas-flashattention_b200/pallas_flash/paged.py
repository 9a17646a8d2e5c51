"""Paged attention (block-table KV cache) on B200.

Drop-in for ``src/pallas_flash/paged.py`` of the reference.  Layout:

    k_pages / v_pages : [num_pages, num_kv_heads, page_size, head_dim]
    block_tables      : [batch, pages_per_seq]  int32  (logical -> physical page)
    context_lens      : [batch]                 int32  (valid tokens per sequence)

The decode kernel resolves ``block_tables[b, p]`` on the device while it
streams pages into shared memory with bulk copies; pages at or past
``context_lens[b]`` are never read (so, unlike the reference, unused trailing
table entries need not be valid page ids).  One CTA serves all query heads of
a kv head, so each page crosses HBM once per step.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

__all__ = ["paged_flash_attention", "paged_prefill_attention", "init_paged_cache", "write_to_paged_cache",
           "write_to_paged_cache_batch", "rope_write_to_paged_cache_batch", "gather_paged"]


def paged_flash_attention(
    q: torch.Tensor,
    k_pages: torch.Tensor,
    v_pages: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    sm_scale: Optional[float] = None,
    interpret: bool = False,
    max_context_len: Optional[int] = None,
) -> torch.Tensor:
    """Single-query attention over a paged KV cache (paged.py:102-192).

    Returns ``[batch, num_heads, 1, head_dim]``.  ``max_context_len`` is an
    optional upper bound of ``context_lens`` (it sizes the split grid; the
    default is the table capacity ``pages_per_seq * page_size``).  A length
    above it raises ``ValueError`` when ``context_lens`` is a host tensor; for
    device lengths the kernel records ``PF_DEV_LEN_OVER_MAX`` in the device
    status word (the keys past the planned splits are then not attended).
    """
    del interpret
    if q.ndim != 4 or q.shape[2] != 1:
        raise ValueError(
            f"paged attention expects q of shape [batch, heads, 1, head_dim], got {tuple(q.shape)}"
        )
    if k_pages.shape != v_pages.shape:
        raise ValueError("k_pages and v_pages must have the same shape")
    batch, num_heads, _, head_dim = q.shape
    num_pages, num_kv_heads, page_size, k_head_dim = k_pages.shape
    if k_head_dim != head_dim:
        raise ValueError("q and pages must share head_dim")
    if num_heads % num_kv_heads != 0:
        raise ValueError(
            f"num_heads ({num_heads}) must be a multiple of num_kv_heads ({num_kv_heads})"
        )
    if block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError(
            f"block_tables must be [batch, pages_per_seq], got {tuple(block_tables.shape)}"
        )
    if tuple(context_lens.shape) != (batch,):
        raise ValueError(f"context_lens must be [batch], got {tuple(context_lens.shape)}")
    if not (q.dtype == k_pages.dtype == v_pages.dtype):
        raise ValueError("q and the page pools must share a dtype")
    _lib.require_cuda(q, k_pages, v_pages)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    dev = q.device
    tables = block_tables.to(device=dev, dtype=torch.int32).contiguous()
    lens = context_lens.to(device=dev, dtype=torch.int32).contiguous()
    pages_per_seq = tables.shape[1]
    cap = pages_per_seq * page_size
    max_len = cap if max_context_len is None else max(1, min(int(max_context_len), cap))
    if max_context_len is not None and context_lens.device.type == "cpu" and context_lens.numel():
        longest = int(context_lens.max())
        if longest > max_len:
            raise ValueError(f"context_lens has a length {longest} above max_context_len {max_len}")
    q, k_pages, v_pages = q.contiguous(), k_pages.contiguous(), v_pages.contiguous()
    out = torch.empty_like(q)
    L = _lib.lib()
    ws = _lib.workspace(
        L.pf_paged_decode_workspace_size(batch, num_heads, num_kv_heads, page_size, max_len, head_dim), dev)
    _lib.check(L.pf_paged_decode(
        q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), tables.data_ptr(), lens.data_ptr(),
        out.data_ptr(), _lib.dtype_code(q.dtype), batch, num_heads, num_kv_heads, num_pages,
        page_size, pages_per_seq, head_dim, max_len, float(sm_scale), ws.data_ptr(), ws.numel(),
        _lib.stream_of(q)))
    return out


def paged_prefill_attention(
    q: torch.Tensor,
    k_pages: torch.Tensor,
    v_pages: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    sm_scale: Optional[float] = None,
    max_context_len: Optional[int] = None,
) -> torch.Tensor:
    """Chunked prefill over a page pool (extends paged.py:102-192 from one query to L).

    ``q``: ``[batch, heads, L, head_dim]``, the last L positions of every
    sequence: row i of sequence b sits at position ``context_lens[b] - L + i``
    and attends causally to keys ``[0, position]`` of that sequence, whose k/v
    (including the chunk's own) are already in the pages.  Returns an array
    shaped like ``q``.  ``max_context_len`` bounds ``context_lens`` (default:
    the table capacity).
    """
    if q.ndim != 4:
        raise ValueError(f"q must be [batch, heads, L, head_dim], got {tuple(q.shape)}")
    if k_pages.shape != v_pages.shape:
        raise ValueError("k_pages and v_pages must have the same shape")
    batch, n_heads, L, head_dim = q.shape
    num_pages, n_kv, page_size, k_head_dim = k_pages.shape
    if k_head_dim != head_dim:
        raise ValueError("q and pages must share head_dim")
    if n_heads % n_kv != 0:
        raise ValueError(f"num_heads ({n_heads}) must be a multiple of num_kv_heads ({n_kv})")
    if block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError(f"block_tables must be [batch, pages_per_seq], got {tuple(block_tables.shape)}")
    if tuple(context_lens.shape) != (batch,):
        raise ValueError(f"context_lens must be [batch], got {tuple(context_lens.shape)}")
    if not (q.dtype == k_pages.dtype == v_pages.dtype):
        raise ValueError("q and the page pools must share a dtype")
    _lib.require_cuda(q, k_pages, v_pages)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    dev = q.device
    tables = block_tables.to(device=dev, dtype=torch.int32).contiguous()
    lens = context_lens.to(device=dev, dtype=torch.int32).contiguous()
    cap = tables.shape[1] * page_size
    max_len = cap if max_context_len is None else max(1, min(int(max_context_len), cap))
    q, k_pages, v_pages = q.contiguous(), k_pages.contiguous(), v_pages.contiguous()
    out = torch.empty_like(q)
    L_ = _lib.lib()
    code = _lib.dtype_code(q.dtype)
    ws = _lib.workspace(L_.pf_paged_prefill_workspace_size(code, batch, n_kv, max_len, head_dim), dev)
    _lib.check(L_.pf_paged_prefill(
        q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), tables.data_ptr(), lens.data_ptr(), out.data_ptr(),
        code, batch, n_heads, n_kv, L, num_pages, page_size, tables.shape[1], head_dim, max_len, float(sm_scale),
        ws.data_ptr(), ws.numel(), _lib.stream_of(q)))
    return out


def init_paged_cache(num_pages: int, num_kv_heads: int, page_size: int, head_dim: int,
                     dtype=torch.float32, device=None):
    """Allocate an empty (zeroed) page pool ``(k_pages, v_pages)`` (paged.py:198-202)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    shape = (num_pages, num_kv_heads, page_size, head_dim)
    return (torch.zeros(shape, dtype=dtype, device=device),
            torch.zeros(shape, dtype=dtype, device=device))


def write_to_paged_cache_batch(k_pages, v_pages, k, v, block_tables, positions):
    """Writes one token per sequence, in place.

    ``k``/``v``: ``[batch, num_kv_heads, 1, head_dim]``; ``block_tables``:
    ``[batch, pages_per_seq]``; ``positions``: ``[batch]`` absolute positions.
    Token b lands in page ``block_tables[b, pos // page_size]`` at offset
    ``pos % page_size``.  Returns ``(k_pages, v_pages)``.
    """
    _lib.require_cuda(k_pages, v_pages, k, v)
    num_pages, n_kv, page_size, head_dim = k_pages.shape
    batch = k.shape[0]
    if k.shape != (batch, n_kv, 1, head_dim) or v.shape != k.shape:
        raise ValueError(f"k/v must be [batch, {n_kv}, 1, {head_dim}], got {tuple(k.shape)}")
    if not (k_pages.is_contiguous() and v_pages.is_contiguous()):
        raise ValueError("page pools must be contiguous to be written in place")
    dev = k_pages.device
    tables = torch.as_tensor(block_tables, dtype=torch.int32, device=dev).reshape(batch, -1).contiguous()
    pos = torch.as_tensor(positions, dtype=torch.int32, device=dev).reshape(batch).contiguous()
    kk = k.to(k_pages.dtype).contiguous()
    vv = v.to(v_pages.dtype).contiguous()
    _lib.check(_lib.lib().pf_paged_write(
        k_pages.data_ptr(), v_pages.data_ptr(), kk.data_ptr(), vv.data_ptr(), tables.data_ptr(),
        pos.data_ptr(), _lib.dtype_code(k_pages.dtype), batch, n_kv, num_pages, page_size,
        tables.shape[1], head_dim, _lib.stream_of(k_pages)))
    return k_pages, v_pages


def rope_write_to_paged_cache_batch(q, k, v, k_pages, v_pages, cos, sin, block_tables, positions,
                                    rope_positions):
    """The step before decode attention in one launch: RoPE on the token's q and k, then the k/v page write.

    ``q``: ``[batch, num_heads, 1, head_dim]``, rotated in place (and returned);
    ``k``/``v``: ``[batch, num_kv_heads, 1, head_dim]``; ``cos``/``sin``:
    ``[rows, head_dim]`` tables, row ``rope_positions[b]`` (clamped into range)
    rotating sequence b; rotated k and v land like
    ``write_to_paged_cache_batch`` at slot ``positions[b]``.  Equivalent to
    ``apply_rope`` on q and k (model.py:338-342) followed by the page write
    (paged.py:205-223), with the rotation in fp32 and one rounding.
    """
    _lib.require_cuda(q, k, v, k_pages, v_pages, cos, sin)
    batch, n_heads, one, head_dim = q.shape
    num_pages, n_kv, page_size, _ = k_pages.shape
    if one != 1 or k.shape != (batch, n_kv, 1, head_dim) or v.shape != k.shape:
        raise ValueError("q must be [batch, heads, 1, D] and k/v [batch, num_kv_heads, 1, D] of the pools")
    if tuple(cos.shape) != tuple(sin.shape) or cos.shape[1] != head_dim:
        raise ValueError(f"cos/sin must be [rows, {head_dim}]")
    if not (k_pages.is_contiguous() and v_pages.is_contiguous()):
        raise ValueError("page pools must be contiguous to be written in place")
    dev = k_pages.device
    tables = torch.as_tensor(block_tables, dtype=torch.int32, device=dev).reshape(batch, -1).contiguous()
    pos = torch.as_tensor(positions, dtype=torch.int32, device=dev).reshape(batch).contiguous()
    rpos = torch.as_tensor(rope_positions, dtype=torch.int32, device=dev).reshape(batch).contiguous()
    if q.dtype != k_pages.dtype or not q.is_contiguous():
        q = q.to(k_pages.dtype).contiguous()
    kk = k.to(k_pages.dtype).contiguous()
    vv = v.to(v_pages.dtype).contiguous()
    sin = sin.to(cos.dtype)
    _lib.check(_lib.lib().pf_rope_paged_write(
        q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), kk.data_ptr(), vv.data_ptr(),
        cos.contiguous().data_ptr(), sin.contiguous().data_ptr(), _lib.dtype_code(cos.dtype), cos.shape[0],
        tables.data_ptr(), pos.data_ptr(), rpos.data_ptr(), _lib.dtype_code(q.dtype), batch, n_heads, n_kv,
        num_pages, page_size, tables.shape[1], head_dim, _lib.stream_of(q)))
    return q


def rope_write_to_paged_cache_qkv(qkv, num_heads: int, k_pages, v_pages, cos, sin, block_tables, positions,
                                  rope_positions):
    """``rope_write_to_paged_cache_batch`` on one fused projection: ``qkv`` is
    ``[batch, 1, (num_heads + 2 * num_kv_heads) * head_dim]`` (q heads, then k heads, then v
    heads, as ``h @ [W_q | W_k | W_v]`` gives them).  Returns the rotated q as a new
    ``[batch, num_heads, 1, head_dim]`` tensor; k and v land in the pages.  One launch, no
    split/copy of the projection."""
    _lib.require_cuda(qkv, k_pages, v_pages, cos, sin)
    num_pages, n_kv, page_size, head_dim = k_pages.shape
    batch = qkv.shape[0]
    width = (num_heads + 2 * n_kv) * head_dim
    if qkv.dim() != 3 or qkv.shape[1] != 1 or qkv.shape[2] != width:
        raise ValueError(f"qkv must be [batch, 1, {width}] for {num_heads}/{n_kv} heads of {head_dim}")
    if qkv.dtype != k_pages.dtype:
        raise ValueError("qkv and the page pools must have the same dtype")
    if tuple(cos.shape) != tuple(sin.shape) or cos.shape[1] != head_dim:
        raise ValueError(f"cos/sin must be [rows, {head_dim}]")
    if not (k_pages.is_contiguous() and v_pages.is_contiguous()):
        raise ValueError("page pools must be contiguous to be written in place")
    dev = k_pages.device
    tables = torch.as_tensor(block_tables, dtype=torch.int32, device=dev).reshape(batch, -1).contiguous()
    pos = torch.as_tensor(positions, dtype=torch.int32, device=dev).reshape(batch).contiguous()
    rpos = torch.as_tensor(rope_positions, dtype=torch.int32, device=dev).reshape(batch).contiguous()
    src = qkv.contiguous()
    q = torch.empty((batch, num_heads, 1, head_dim), dtype=qkv.dtype, device=dev)
    sin = sin.to(cos.dtype)
    _lib.check(_lib.lib().pf_rope_paged_write_qkv(
        src.data_ptr(), width, q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
        cos.contiguous().data_ptr(), sin.contiguous().data_ptr(), _lib.dtype_code(cos.dtype), cos.shape[0],
        tables.data_ptr(), pos.data_ptr(), rpos.data_ptr(), _lib.dtype_code(q.dtype), batch, num_heads, n_kv,
        num_pages, page_size, tables.shape[1], head_dim, _lib.stream_of(src)))
    return q


def write_to_paged_cache(k_pages, v_pages, k, v, block_table, position: int):
    """Write one token's K/V into the page holding ``position`` (paged.py:205-223).

    ``k``/``v``: ``[1, num_kv_heads, 1, head_dim]``; ``block_table``:
    ``[pages_per_seq]``.  The pools are updated in place and returned, so the
    reference's functional ``k_pages, v_pages = write_to_paged_cache(...)``
    idiom works unchanged.  A physical page id outside the pool is clamped
    (``dynamic_update_slice`` semantics); a logical page beyond the table
    raises ``IndexError`` like indexing a jax array with a static int.
    """
    page_size = k_pages.shape[2]
    logical_page = int(position) // page_size
    n_entries = int(block_table.shape[0]) if hasattr(block_table, "shape") else len(block_table)
    if not 0 <= logical_page < n_entries:
        raise IndexError(
            f"index {logical_page} is out of bounds for axis 0 with size {n_entries}")
    return write_to_paged_cache_batch(k_pages, v_pages, k, v,
                                      torch.as_tensor(block_table).reshape(1, -1),
                                      [int(position)])


def gather_paged(pages: torch.Tensor, block_tables: torch.Tensor) -> torch.Tensor:
    """Contiguous ``[batch, num_kv_heads, pages_per_seq*page_size, head_dim]`` view of a pool.

    Byte-exact materialisation of the block-table index map
    (``(block_tables[b, p], h, :, :)``, paged.py:158-159); out-of-range page
    ids are flagged in the device status word instead of being read.
    """
    _lib.require_cuda(pages)
    num_pages, n_kv, page_size, head_dim = pages.shape
    tables = block_tables.to(device=pages.device, dtype=torch.int32).contiguous()
    batch, pps = tables.shape
    out = torch.empty((batch, n_kv, pps * page_size, head_dim), dtype=pages.dtype, device=pages.device)
    _lib.check(_lib.lib().pf_paged_gather(
        pages.contiguous().data_ptr(), tables.data_ptr(), out.data_ptr(),
        _lib.dtype_code(pages.dtype), batch, n_kv, num_pages, page_size, pps, head_dim,
        _lib.stream_of(pages)))
    return out
