"""CPU parity oracle for the pallas_flash hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or as the timed
CPU restatement of the reference; no product code path imports it.

It restates, in numpy, the algorithm of the reference
(aabhimittal/TPU-Native-Pallas-FlashAttention, JAX/Pallas):

* ``reference_attention``  -- src/pallas_flash/reference.py:22-66 (naive
  softmax(QK^T*s)V, GQA by head repetition, causal mask -1e30, fp32 softmax),
  extended with the kernels' ``kv_len`` key mask (flash_attention.py:114-120);
* ``attention_vjp``        -- the gradient the reference's tests compare against
  (``jax.grad`` through reference_attention, tests/test_backward.py:107-119),
  in closed form: the formulas of flash_attention.py:233-244 / the notebook's
  manual_bwd, with the GQA group-sum of flash_attention.py:433-436;
* ``precompute_rope`` / ``apply_rope`` -- src/pallas_flash/model.py:41-67;
* ``gather_contiguous`` / ``paged_attention`` -- tests/test_paged.py:25-28 and
  the block-table index map of src/pallas_flash/paged.py:158-159;
* ``ring_slots`` -- src/pallas_flash/model.py:434-449, :475-476;
* ``tiny_llama_forward`` -- src/pallas_flash/model.py:34-140;
  ``tiny_llama_generate`` -- the fixed-cache and ring-cache greedy loops of
  model.py:307-386 and :406-531.

Parity pinning: JAX is not installed here or on the GPU hosts, but the
reference's own source runs under a numpy stand-in for the jax names it uses
(tests/golden/jax_numpy_shim.py; ``pallas_call`` executes each Pallas kernel
body grid point by grid point, as interpret mode does).
tests/golden/make_reference_golden.py executes the UNMODIFIED reference files
-- the forward/backward/decode/fused-RoPE/paged Pallas kernels, the naive
``reference_attention``, the page helpers and the model's ``forward`` /
``generate`` / ``generate_cached`` / ``generate_streaming`` -- with float32
widened to float64, and stores their outputs in
tests/golden/reference_golden.npz.  tests/test_reference_golden.py checks this
oracle against those outputs (float32 rounding), and
tests/test_reference_golden_gpu.py checks the CUDA kernels against them.
Further pins: the reference tests' known-answer cases (uniform attention over
all-ones K/V returns exactly 1.0, NaN beyond the valid length never leaks,
shared pages give identical rows, key-order invariance, ring_kv_len values)
and tests/golden/attention_cases.npz (float64 torch autograd of the same math,
tests/golden/make_golden.py).  Bit-level rounding of the TPU kernels is not
reproduced (parity for floating point is by tolerance).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import numpy as np

NEG_INF = -1e30  # reference.py:62, flash_attention.py:50


def _repeat_kv(x: np.ndarray, n_heads: int) -> np.ndarray:
    rep = n_heads // x.shape[1]
    return np.repeat(x, rep, axis=1) if rep != 1 else x


def _mask(sq: int, sk: int, causal: bool, kv_len: Optional[int]) -> np.ndarray:
    """True where a (query, key) pair is visible."""
    qp = np.arange(sq)[:, None]
    kp = np.arange(sk)[None, :]
    m = np.ones((sq, sk), dtype=bool)
    if kv_len is not None:
        m &= kp < kv_len
    if causal:
        m &= qp >= kp
    return m


def _softmax(s: np.ndarray) -> np.ndarray:
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    return e / e.sum(axis=-1, keepdims=True)


def reference_attention(q, k, v, *, causal: bool = False, sm_scale: Optional[float] = None,
                        kv_len: Optional[int] = None, dtype=np.float64) -> np.ndarray:
    """Naive attention in ``dtype`` arithmetic (reference.py:45-66 + kv_len mask).

    Inputs are numpy arrays (any float dtype, bf16 values already widened).
    Rows with no visible key return 0 (the kernels' finalize rule,
    flash_attention.py:150-159).  Keys past ``kv_len`` are excluded before any
    arithmetic, so NaN there cannot leak.
    """
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    head_dim = q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    sk = k.shape[2]
    if kv_len is not None:
        k = k[:, :, :kv_len]
        v = v[:, :, :kv_len]
        sk = kv_len
    k = _repeat_kv(k, q.shape[1])
    v = _repeat_kv(v, q.shape[1])
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * dtype(sm_scale)
    vis = _mask(q.shape[2], sk, causal, None)
    s = np.where(vis, s, dtype(NEG_INF))
    p = _softmax(s)
    out = np.einsum("bhqk,bhkd->bhqd", p, v)
    empty = ~vis.any(axis=-1)
    if empty.any():
        out[:, :, empty, :] = 0
    return out


def attention_lse(q, k, v, *, causal=False, sm_scale=None, kv_len=None, dtype=np.float64):
    """Row log-sum-exp ``[B, H, Sq, 1]`` of the scaled, masked scores (0 for empty rows)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    if kv_len is not None:
        k = k[:, :, :kv_len]
    k = _repeat_kv(k, q.shape[1])
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * dtype(sm_scale)
    vis = _mask(q.shape[2], k.shape[2], causal, None)
    s = np.where(vis, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, 0)
    lse = m_safe + np.log(np.exp(s - m_safe).sum(axis=-1, keepdims=True))
    return np.where(np.isfinite(m), lse, 0.0)


def attention_vjp(q, k, v, do, *, causal=False, sm_scale=None, kv_len=None, dtype=np.float64):
    """Gradients ``(dq, dk, dv)`` of ``sum(reference_attention(q,k,v) * do)``.

    Closed form of the softmax-attention VJP (flash_attention.py:233-244):
    ``dv = P^T dO``, ``dP = dO V^T``, ``dS = P (dP - rowsum(dO*O))``,
    ``dq = s dS K``, ``dk = s dS^T Q``; dk/dv summed over each GQA group.
    Keys at or past ``kv_len`` get zero gradient.
    """
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    do = np.asarray(do, dtype)
    B, H, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    kl = Sk if kv_len is None else kv_len
    kr = _repeat_kv(k[:, :, :kl], H)
    vr = _repeat_kv(v[:, :, :kl], H)
    s = np.einsum("bhqd,bhkd->bhqk", q, kr) * dtype(sm_scale)
    vis = _mask(Sq, kl, causal, None)
    s = np.where(vis, s, dtype(NEG_INF))
    p = _softmax(s)
    p = np.where(vis, p, 0)
    o = np.einsum("bhqk,bhkd->bhqd", p, vr)
    dv_h = np.einsum("bhqk,bhqd->bhkd", p, do)
    dp = np.einsum("bhqd,bhkd->bhqk", do, vr)
    delta = (o * do).sum(axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = np.einsum("bhqk,bhkd->bhqd", ds, kr) * dtype(sm_scale)
    dk_h = np.einsum("bhqk,bhqd->bhkd", ds, q) * dtype(sm_scale)
    g = H // Hkv
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dk[:, :, :kl] = dk_h.reshape(B, Hkv, g, kl, D).sum(axis=2)
    dv[:, :, :kl] = dv_h.reshape(B, Hkv, g, kl, D).sum(axis=2)
    return dq, dk, dv


# --------------------------------------------------------------------------- #
# RoPE (model.py:41-67, fused_rope.py:43-50)
# --------------------------------------------------------------------------- #
def precompute_rope(seq_len: int, head_dim: int, theta: float, dtype=np.float32):
    half = head_dim // 2
    inv_freq = 1.0 / (np.float32(theta) ** (np.arange(0, half, dtype=np.float32) / np.float32(half)))
    pos = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(pos, inv_freq).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(dtype), np.sin(emb).astype(dtype)


def rotate_half(x: np.ndarray) -> np.ndarray:
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(x, cos, sin):
    """``x * cos + rotate_half(x) * sin`` with tables ``[seq, head_dim]`` broadcast over B, H."""
    return x * cos[None, None] + rotate_half(x) * sin[None, None]


# --------------------------------------------------------------------------- #
# Paged cache (tests/test_paged.py:16-28, paged.py:158-159, :205-223)
# --------------------------------------------------------------------------- #
def gather_contiguous(pages: np.ndarray, table_row: Sequence[int], pages_per_seq: int,
                      length: int) -> np.ndarray:
    """Sequence KV ``[Hkv, length, D]`` rebuilt from its pages in table order."""
    parts = [pages[int(table_row[p])] for p in range(pages_per_seq)]
    return np.concatenate(parts, axis=1)[:, :length]


def paged_attention(q, k_pages, v_pages, block_tables, context_lens, *, sm_scale=None,
                    dtype=np.float64):
    """Reference result of paged decode: per sequence, attention over its gathered prefix."""
    q = np.asarray(q)
    out = np.zeros(q.shape, dtype)
    pps = block_tables.shape[1]
    for b, length in enumerate(np.asarray(context_lens).tolist()):
        if length == 0:
            continue
        kc = gather_contiguous(k_pages, block_tables[b], pps, length)[None]
        vc = gather_contiguous(v_pages, block_tables[b], pps, length)[None]
        out[b:b + 1] = reference_attention(q[b:b + 1], kc, vc, sm_scale=sm_scale, dtype=dtype)
    return out


def paged_write(k_pages, v_pages, k, v, block_table, position: int):
    """In-place single-token write at page ``block_table[pos // ps]``, offset ``pos % ps``.

    The physical page index is clamped into the pool like dynamic_update_slice.
    """
    ps = k_pages.shape[2]
    lp, off = divmod(int(position), ps)
    page = min(max(int(block_table[lp]), 0), k_pages.shape[0] - 1)
    k_pages[page, :, off] = k[0, :, 0]
    v_pages[page, :, off] = v[0, :, 0]


def ring_slots(start: int, stop: int, capacity: int) -> np.ndarray:
    """Ring slots of absolute positions ``[start, stop)`` (model.py:437)."""
    return np.arange(start, stop) % capacity


def ring_kv_len(total_tokens: int, capacity: int) -> int:
    return min(total_tokens, capacity)


# --------------------------------------------------------------------------- #
# Tiny LLaMA forward (model.py:34-140), fp32 numpy
# --------------------------------------------------------------------------- #
def rms_norm(x, w, eps):
    x = x.astype(np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(var + np.float32(eps)) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def tiny_llama_forward(params: dict, tokens: np.ndarray, cfg) -> np.ndarray:
    """Logits ``[batch, seq, vocab]`` of the reference model on numpy fp32 parameters."""
    b, seq = tokens.shape
    x = params["embed"][tokens].astype(np.float32)
    cos, sin = precompute_rope(seq, cfg.head_dim, cfg.rope_theta)
    for layer in params["layers"]:
        h = rms_norm(x, layer["attn_norm"], cfg.rms_norm_eps)

        def split(t, n):
            return t.reshape(b, seq, n, cfg.head_dim).transpose(0, 2, 1, 3)

        q = apply_rope(split(h @ layer["wq"], cfg.n_heads), cos, sin)
        k = apply_rope(split(h @ layer["wk"], cfg.n_kv_heads), cos, sin)
        v = split(h @ layer["wv"], cfg.n_kv_heads)
        a = reference_attention(q, k, v, causal=True, dtype=np.float32)
        x = x + a.transpose(0, 2, 1, 3).reshape(b, seq, cfg.dim) @ layer["wo"]
        h = rms_norm(x, layer["ffn_norm"], cfg.rms_norm_eps)
        x = x + (_silu(h @ layer["w_gate"]) * (h @ layer["w_up"])) @ layer["w_down"]
    x = rms_norm(x, params["final_norm"], cfg.rms_norm_eps)
    return x @ params["lm_head"]


def tiny_llama_generate(params: dict, prompts: np.ndarray, max_new_tokens: int, cfg,
                        window: Optional[int] = None) -> np.ndarray:
    """Greedy generation with a KV cache, numpy fp32.

    ``window=None``: the fixed cache of ``generate_cached`` (model.py:307-386,
    capacity prompt + new tokens); ``window=W``: the ring cache of
    ``generate_streaming`` (model.py:406-531): the prompt is attended in full,
    its last ``min(prompt, W)`` K/V rows are kept at slots ``pos % W``, and each
    decode step writes slot ``pos % W`` and attends the ``min(pos + 1, W)``
    live slots.  Returns ``[batch, prompt + max_new_tokens]`` token ids.
    """
    b, seq = prompts.shape
    hd, nkv = cfg.head_dim, cfg.n_kv_heads
    cap = seq + max_new_tokens if window is None else window
    total = seq + max_new_tokens
    cos_all, sin_all = precompute_rope(total, hd, cfg.rope_theta)

    def split(t, n, length):
        return t.reshape(b, length, n, hd).transpose(0, 2, 1, 3)

    caches = [(np.zeros((b, nkv, cap, hd), np.float32), np.zeros((b, nkv, cap, hd), np.float32))
              for _ in params["layers"]]
    # prefill
    x = params["embed"][prompts].astype(np.float32)
    cos, sin = cos_all[:seq], sin_all[:seq]
    keep = min(seq, cap)
    slots = np.arange(seq - keep, seq) % cap
    for layer, (kc, vc) in zip(params["layers"], caches):
        h = rms_norm(x, layer["attn_norm"], cfg.rms_norm_eps)
        q = apply_rope(split(h @ layer["wq"], cfg.n_heads, seq), cos, sin)
        k = apply_rope(split(h @ layer["wk"], nkv, seq), cos, sin)
        v = split(h @ layer["wv"], nkv, seq)
        kc[:, :, slots] = k[:, :, seq - keep:]
        vc[:, :, slots] = v[:, :, seq - keep:]
        a = reference_attention(q, k, v, causal=True, dtype=np.float32)
        x = x + a.transpose(0, 2, 1, 3).reshape(b, seq, cfg.dim) @ layer["wo"]
        h = rms_norm(x, layer["ffn_norm"], cfg.rms_norm_eps)
        x = x + (_silu(h @ layer["w_gate"]) * (h @ layer["w_up"])) @ layer["w_down"]
    logits = rms_norm(x, params["final_norm"], cfg.rms_norm_eps)[:, -1] @ params["lm_head"]
    out = [prompts, np.argmax(logits, axis=-1)[:, None]]
    for i in range(max_new_tokens - 1):
        pos = seq + i
        slot, live = pos % cap, min(pos + 1, cap)
        x = params["embed"][out[-1]].astype(np.float32)
        cos, sin = cos_all[pos:pos + 1], sin_all[pos:pos + 1]
        for layer, (kc, vc) in zip(params["layers"], caches):
            h = rms_norm(x, layer["attn_norm"], cfg.rms_norm_eps)
            q = apply_rope(split(h @ layer["wq"], cfg.n_heads, 1), cos, sin)
            kc[:, :, slot] = apply_rope(split(h @ layer["wk"], nkv, 1), cos, sin)[:, :, 0]
            vc[:, :, slot] = split(h @ layer["wv"], nkv, 1)[:, :, 0]
            a = reference_attention(q, kc, vc, kv_len=live, dtype=np.float32)
            x = x + a.transpose(0, 2, 1, 3).reshape(b, 1, cfg.dim) @ layer["wo"]
            h = rms_norm(x, layer["ffn_norm"], cfg.rms_norm_eps)
            x = x + (_silu(h @ layer["w_gate"]) * (h @ layer["w_up"])) @ layer["w_down"]
        logits = rms_norm(x, params["final_norm"], cfg.rms_norm_eps)[:, -1] @ params["lm_head"]
        out.append(np.argmax(logits, axis=-1)[:, None])
    return np.concatenate(out, axis=1)


# --------------------------------------------------------------------------- #
# bf16 helpers (numpy has no bfloat16)
# --------------------------------------------------------------------------- #
def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned widened to float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.nan
    return out
