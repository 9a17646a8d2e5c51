"""Tiny LLaMA decoder on the B200 attention kernels.

Drop-in for ``src/pallas_flash/model.py`` of the reference: the same functions,
parameter pytree (a dict with ``embed``, ``layers`` [list of dicts],
``final_norm``, ``lm_head``) and greedy generation loops, on CUDA tensors.
Attention goes through this package's kernels (``flash_attention`` for
prefill/forward, ``flash_attention_decode`` for decode steps).  The dense layers
(projections, SwiGLU, lm_head) of the prefill and of the lm_head are PyTorch
matmuls (cuBLAS), which the reference likewise leaves to its compiler; in a
16-bit decode step of at most 16 sequences the four per-block projections run
through ``pf_rows_linear`` with the RMSNorm before them, the residual add after
them and the SwiGLU activation between them folded in, and RoPE plus the K/V
cache write in the q/k/v projection's epilogue (5 launches per block with the
attention, where the unfused chain takes 9).

Differences that keep behaviour but suit the GPU:
* KV caches are preallocated and written **in place** by the cache-write
  kernel; ``decode_step`` / ``ring_decode_step`` return the same (mutated)
  cache list, so the reference's ``logits, cache = decode_step(...)`` idiom is
  unchanged;
* RoPE tables are computed once per (length, dtype, device) and sliced, instead
  of being rebuilt for ``pos + 1`` rows every step (model.py:240-243);
* ``init_params`` takes an integer seed (or a ``torch.Generator``) where the
  reference takes a ``jax.random.PRNGKey``.
"""

from __future__ import annotations

import weakref
from typing import Any, Dict, List, Optional

import torch

from . import _lib
from .config import ModelConfig
from .flash_attention import flash_attention, flash_attention_decode
from .paged import paged_flash_attention, rope_write_to_paged_cache_qkv

Params = Dict[str, Any]
Cache = list  # per-layer list of {"k": [b, n_kv, cache_size, d], "v": same}


# --------------------------------------------------------------------------- #
# Building blocks (model.py:34-74)
# --------------------------------------------------------------------------- #
def _add_rms_norm_kernel(x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                         eps: float):
    """``x' = x + residual`` (``x' = x`` when ``residual`` is None) and ``rms_norm(x')``, as
    ``(x', h)`` from one kernel launch (``pf_add_rms_norm``).  The sum is rounded to
    ``x.dtype`` as the unfused ``x + residual`` rounds it; the norm follows model.py:34-38
    in fp32 (``weight`` is taken in ``x.dtype``)."""
    _lib.require_cuda(x, weight)
    dim = x.shape[-1]
    if weight.numel() != dim:
        raise ValueError(f"norm weight has {weight.numel()} elements, expected {dim}")
    xc = x.contiguous()
    w = weight.to(x.dtype).contiguous()
    h = torch.empty_like(xc)
    if residual is None:
        x_out, r = xc, None
    else:
        if residual.shape != x.shape:
            raise ValueError(f"residual shape {tuple(residual.shape)} != x shape {tuple(x.shape)}")
        r = residual.to(x.dtype).contiguous()
        x_out = torch.empty_like(xc)
    _lib.check(_lib.lib().pf_add_rms_norm(xc.data_ptr(), _lib.ptr(r), w.data_ptr(),
                                          x_out.data_ptr() if r is not None else None, h.data_ptr(),
                                          _lib.dtype_code(x.dtype), xc.numel() // dim, dim, float(eps),
                                          _lib.stream_of(x)))
    return x_out, h


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


class _RmsNormFn(torch.autograd.Function):
    """rms_norm with the kernel forward and the closed-form fp32 gradient:
    with r = rsqrt(mean(x^2) + eps) and g = dh * w,
    dx = r * g - x * r^3 * mean(g * x),  dw = sum over rows of dh * x * r."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        return _add_rms_norm_kernel(x, None, weight, eps)[1]

    @staticmethod
    def backward(ctx, dh):
        x, w = ctx.saved_tensors
        xf, gf = x.float(), dh.float() * w.float()
        r = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + ctx.eps)
        dx = r * gf - xf * r.pow(3) * (gf * xf).mean(dim=-1, keepdim=True)
        dw = (dh.float() * xf * r).reshape(-1, x.shape[-1]).sum(dim=0)
        return dx.to(x.dtype), dw.to(w.dtype), None


def add_rms_norm(x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                 eps: float):
    """``x' = x + residual`` (``x' = x`` when ``residual`` is None) and ``rms_norm(x')``, as
    ``(x', h)``: one kernel launch (``pf_add_rms_norm``) for inference.  When a gradient is
    needed, the sum is a differentiable tensor add and the norm runs the same kernel inside
    an autograd function (closed-form backward)."""
    if _needs_grad(x, residual, weight):
        xs = x if residual is None else x + residual.to(x.dtype)
        return xs, _RmsNormFn.apply(xs, weight.to(x.dtype), float(eps))
    return _add_rms_norm_kernel(x, residual, weight, eps)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Root-mean-square layer norm (LLaMA-style, no mean subtraction), one kernel launch."""
    return add_rms_norm(x, None, weight, eps)[1]


def precompute_rope(seq_len: int, head_dim: int, theta: float, device=None):
    """cos/sin tables ``[seq_len, head_dim]`` (fp32): ``emb = [f, f]``, ``f = pos * theta^(-i/half)``."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32, device=device) / half))
    pos = torch.arange(seq_len, dtype=torch.float32, device=device)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return torch.cos(emb), torch.sin(emb)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Apply rotary embeddings to ``x`` ``[batch, heads, seq, head_dim]`` (tables ``[seq, head_dim]``)."""
    return x * cos[None, None] + _rotate_half(x) * sin[None, None]


def _silu_mul_kernel(gate: torch.Tensor, up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(gate) * up`` in one launch (``pf_silu_mul``); silu is rounded to the tensor
    dtype before the product, as in the unfused expression.  With ``up`` None, ``gate``
    is one fused ``[..., 2F]`` projection whose halves are the gate and the up values."""
    _lib.require_cuda(gate)
    if up is None:
        g = gate.contiguous()
        cols = g.shape[-1] // 2
        if g.shape[-1] != 2 * cols:
            raise ValueError("silu_mul: a fused projection must have an even last dimension")
        gp, up_ptr, stride = g.data_ptr(), g.data_ptr() + cols * g.element_size(), 2 * cols
        out_shape = (*g.shape[:-1], cols)
    else:
        _lib.require_cuda(up)
        if gate.shape != up.shape or gate.dtype != up.dtype:
            raise ValueError("silu_mul: gate and up must have the same shape and dtype")
        g, u = gate.contiguous(), up.contiguous()
        cols = g.shape[-1]
        gp, up_ptr, stride = g.data_ptr(), u.data_ptr(), cols
        out_shape = g.shape
    out = torch.empty(out_shape, dtype=g.dtype, device=g.device)
    rows = out.numel() // cols if cols else 0
    _lib.check(_lib.lib().pf_silu_mul(gp, up_ptr, out.data_ptr(), _lib.dtype_code(g.dtype), rows, cols, stride,
                                      _lib.stream_of(g)))
    return out


class _SiluMulFn(torch.autograd.Function):
    """silu(g) * u with the kernel forward; with s = sigmoid(g):
    dg = dout * u * s * (1 + g * (1 - s)),  du = dout * g * s (fp32)."""

    @staticmethod
    def forward(ctx, g, u):
        ctx.save_for_backward(g, u)
        return _silu_mul_kernel(g, u)

    @staticmethod
    def backward(ctx, dout):
        g, u = ctx.saved_tensors
        gf, uf, df = g.float(), u.float(), dout.float()
        sg = torch.sigmoid(gf)
        dg = df * uf * sg * (1 + gf * (1 - sg))
        du = df * gf * sg
        return dg.to(g.dtype), du.to(u.dtype)


def silu_mul(gate: torch.Tensor, up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(gate) * up`` (``pf_silu_mul``); with ``up`` None, ``gate`` is one fused
    ``[..., 2F]`` projection whose halves are the gate and the up values.  Differentiable:
    when a gradient is needed the kernel runs inside an autograd function."""
    if _needs_grad(gate, up):
        if up is None:
            cols = gate.shape[-1] // 2
            gate, up = gate[..., :cols], gate[..., cols:]
        return _SiluMulFn.apply(gate, up)
    return _silu_mul_kernel(gate, up)


# Column-concatenated copies of weight matrices, so that projections sharing an
# input run as one matmul.  An entry is used only while every source tensor is
# alive (weak references) and unmodified (its version counter): the cache never
# changes results, only the launch count.
_FUSED: Dict[tuple, tuple] = {}


def _fused_columns(*ws: torch.Tensor) -> torch.Tensor:
    if _needs_grad(*ws):  # a differentiable concatenation, rebuilt per call
        return torch.cat(ws, dim=1)
    key = tuple(id(w) for w in ws)
    hit = _FUSED.get(key)
    if hit is not None:
        refs, versions, fused = hit
        if all(r() is w for r, w in zip(refs, ws)) and versions == tuple(w._version for w in ws):
            return fused
    if len(_FUSED) > 512:
        for k in [k for k, (refs, _, _) in _FUSED.items() if any(r() is None for r in refs)]:
            del _FUSED[k]
    fused = torch.cat(ws, dim=1)
    _FUSED[key] = (tuple(weakref.ref(w) for w in ws), tuple(w._version for w in ws), fused)
    return fused


def swiglu_mlp(x, w_gate, w_up, w_down):
    """SwiGLU feed-forward: ``(silu(x W_gate) * (x W_up)) W_down``; the two input
    projections run as one matmul over ``[W_gate | W_up]``."""
    return silu_mul(x @ _fused_columns(w_gate, w_up)) @ w_down


_FUSED_T: Dict[tuple, tuple] = {}


def _fused_rows(*ws: torch.Tensor) -> torch.Tensor:
    """``[W_1 | W_2 | ...]^T`` as a contiguous ``[out_features, in_features]`` tensor, the
    weight layout of ``pf_rows_linear``; built once per set of weights (and rebuilt when
    one of them is modified in place)."""
    key = tuple(id(w) for w in ws)
    hit = _FUSED_T.get(key)
    if hit is not None:
        refs, versions, fused = hit
        if all(r() is w for r, w in zip(refs, ws)) and versions == tuple(w._version for w in ws):
            return fused
    if len(_FUSED_T) > 512:
        for k in [k for k, (refs, _, _) in _FUSED_T.items() if any(r() is None for r in refs)]:
            del _FUSED_T[k]
    with torch.no_grad():
        fused = torch.cat(ws, dim=1).t().contiguous()
    _FUSED_T[key] = (tuple(weakref.ref(w) for w in ws), tuple(w._version for w in ws), fused)
    return fused


def _rows_linear(x: torch.Tensor, wt: torch.Tensor, mode: int, norm: Optional[torch.Tensor] = None,
                 eps: float = 0.0, residual: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``pf_rows_linear`` on ``x`` [M <= 16, K]: mode 0 ``norm?(x) @ W``, 1 ``residual + x @ W``,
    2 ``silu(norm?(x) @ W_gate) * (norm?(x) @ W_up)`` with ``wt = [W_gate | W_up]^T``."""
    M, K = x.shape
    N = wt.shape[0] // (2 if mode == 2 else 1)
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().pf_rows_linear(
        x.data_ptr(), _lib.ptr(norm), float(eps), wt.data_ptr(), _lib.ptr(residual), y.data_ptr(),
        _lib.dtype_code(x.dtype), M, K, N, mode, _lib.stream_of(x)))
    return y


def _qkv_rope_write(x: torch.Tensor, layer: Params, norm: torch.Tensor, eps: float, cfg: ModelConfig,
                    k_pages, v_pages, cos, sin, table, slots, rope_rows) -> torch.Tensor:
    """The normed q/k/v projection of one token per sequence with RoPE and the K/V cache
    write folded in (``pf_rows_linear_rope_write``, one launch); returns the rotated q
    ``[batch, n_heads, 1, head_dim]``.  The fixed / ring cache is addressed as a pool of
    one page per sequence, as ``rope_write_to_paged_cache_qkv`` does."""
    wt = _fused_rows(layer["wq"], layer["wk"], layer["wv"])
    if cfg.head_dim % 32 != 0:
        qkv = _rows_linear(x, wt, 0, norm=norm, eps=eps)
        return rope_write_to_paged_cache_qkv(qkv.reshape(x.shape[0], 1, -1), cfg.n_heads, k_pages, v_pages, cos,
                                             sin, table, slots, rope_rows)
    batch, K = x.shape
    num_pages, n_kv, page_size, head_dim = k_pages.shape
    q = torch.empty((batch, cfg.n_heads, 1, head_dim), dtype=x.dtype, device=x.device)
    sin = sin.to(cos.dtype)
    _lib.check(_lib.lib().pf_rows_linear_rope_write(
        x.data_ptr(), norm.data_ptr(), float(eps), wt.data_ptr(), q.data_ptr(), k_pages.data_ptr(),
        v_pages.data_ptr(), cos.contiguous().data_ptr(), sin.contiguous().data_ptr(), _lib.dtype_code(cos.dtype),
        cos.shape[0], table.data_ptr(), slots.data_ptr(), rope_rows.data_ptr(), _lib.dtype_code(x.dtype), batch, K,
        cfg.n_heads, n_kv, num_pages, page_size, table.shape[1], head_dim, _lib.stream_of(x)))
    return q


def _fused_decode_ok(params: Params, cfg: ModelConfig, batch: int, dtype) -> bool:
    """Whether a decode step can run its projections through ``pf_rows_linear`` (16-bit
    weights, at most 16 rows, dimensions its tiles divide).  The eager step and the graph
    step take the same choice, so their tokens stay identical."""
    if dtype not in (torch.bfloat16, torch.float16) or not 1 <= batch <= 16:
        return False
    if torch.is_grad_enabled() and any(t.requires_grad for t in (params["embed"], params["lm_head"])):
        return False
    width = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    fits = lambda k: k % 32 == 0 and 32 <= k <= 2048  # noqa: E731
    return (fits(cfg.dim) and fits(cfg.ffn_hidden) and width % 32 == 0 and cfg.dim % 32 == 0
            and cfg.ffn_hidden % 16 == 0 and cfg.vocab_size % 32 == 0
            and params["embed"].dtype == dtype and params["lm_head"].dtype == dtype)


_ROPE_CACHE: Dict[tuple, tuple] = {}


def _rope_slice(pos_start: int, length: int, cfg: ModelConfig, dtype, device=None):
    """cos/sin tables for absolute positions ``[pos_start, pos_start+length)`` (model.py:240-243)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    need = pos_start + length
    key = (cfg.head_dim, float(cfg.rope_theta), dtype, str(device))
    ent = _ROPE_CACHE.get(key)
    if ent is None or ent[0].shape[0] < need:
        n = max(need, 2 * ent[0].shape[0] if ent is not None else 1024)
        cos, sin = precompute_rope(n, cfg.head_dim, cfg.rope_theta, device=device)
        ent = (cos.to(dtype), sin.to(dtype))
        _ROPE_CACHE[key] = ent
    return ent[0][pos_start:need], ent[1][pos_start:need]


# --------------------------------------------------------------------------- #
# Decoder block + full model (model.py:80-140)
# --------------------------------------------------------------------------- #
def project_qkv(params: Params, h: torch.Tensor, cfg: ModelConfig):
    """Project normed hidden states to ``[batch, heads, seq, head_dim]`` Q, K, V (pre-RoPE)."""
    batch, seq, _ = h.shape

    def split(t, n_heads):
        return t.reshape(batch, seq, n_heads, cfg.head_dim).transpose(1, 2)

    return (split(h @ params["wq"], cfg.n_heads),
            split(h @ params["wk"], cfg.n_kv_heads),
            split(h @ params["wv"], cfg.n_kv_heads))


def decoder_block(params: Params, x, cos, sin, cfg: ModelConfig, interpret: bool = False):
    """One pre-norm transformer decoder block (causal attention on the B200 kernel)."""
    batch, seq, _ = x.shape
    h = rms_norm(x, params["attn_norm"], cfg.rms_norm_eps)
    q, k, v = project_qkv(params, h, cfg)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    attn = flash_attention(q, k, v, causal=True, block_q=cfg.block_q, block_k=cfg.block_k)
    attn = attn.transpose(1, 2).reshape(batch, seq, cfg.dim)
    x, h = add_rms_norm(x, attn @ params["wo"], params["ffn_norm"], cfg.rms_norm_eps)
    return x + swiglu_mlp(h, params["w_gate"], params["w_up"], params["w_down"])


def forward(params: Params, tokens: torch.Tensor, cfg: ModelConfig, interpret: bool = False):
    """Logits ``[batch, seq, vocab_size]``."""
    seq = tokens.shape[1]
    x = params["embed"][tokens]
    cos, sin = _rope_slice(0, seq, cfg, x.dtype, x.device)
    for layer in params["layers"]:
        x = decoder_block(layer, x, cos, sin, cfg, interpret)
    x = rms_norm(x, params["final_norm"], cfg.rms_norm_eps)
    return x @ params["lm_head"]


# --------------------------------------------------------------------------- #
# Parameter initialization (model.py:146-176)
# --------------------------------------------------------------------------- #
def init_params(key, cfg: ModelConfig, dtype=torch.float32, device=None) -> Params:
    """Random parameters with the reference's shapes and scales (seeded, no training)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    gen = key if isinstance(key, torch.Generator) else torch.Generator().manual_seed(int(key))

    def normal(shape, scale):
        return (torch.randn(shape, generator=gen, dtype=torch.float32) * scale).to(dtype).to(device)

    ones = lambda n: torch.ones((n,), dtype=dtype, device=device)  # noqa: E731
    params: Params = {"embed": normal((cfg.vocab_size, cfg.dim), 0.02)}
    proj = 1.0 / (cfg.dim ** 0.5)
    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "attn_norm": ones(cfg.dim),
            "ffn_norm": ones(cfg.dim),
            "wq": normal((cfg.dim, cfg.dim), proj),
            "wk": normal((cfg.dim, cfg.kv_dim), proj),
            "wv": normal((cfg.dim, cfg.kv_dim), proj),
            "wo": normal((cfg.dim, cfg.dim), proj),
            "w_gate": normal((cfg.dim, cfg.ffn_hidden), proj),
            "w_up": normal((cfg.dim, cfg.ffn_hidden), proj),
            "w_down": normal((cfg.ffn_hidden, cfg.dim), 1.0 / (cfg.ffn_hidden ** 0.5)),
        })
    params["layers"] = layers
    params["final_norm"] = ones(cfg.dim)
    params["lm_head"] = normal((cfg.dim, cfg.vocab_size), proj)
    return params


def _argmax_last(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits[:, -1, :], dim=-1, keepdim=True)


def generate(params: Params, prompt_ids, max_new_tokens: int, cfg: ModelConfig,
             interpret: bool = False):
    """Greedy generation by full recompute each step (model.py:182-207)."""
    tokens = prompt_ids
    for _ in range(max_new_tokens):
        logits = forward(params, tokens, cfg)
        tokens = torch.cat([tokens, _argmax_last(logits).to(tokens.dtype)], dim=1)
    return tokens


# --------------------------------------------------------------------------- #
# KV-cache decoding (model.py:227-386)
# --------------------------------------------------------------------------- #
def _attend(layer: Params, q, k, v, cfg: ModelConfig, interpret: bool, causal: bool):
    batch, _, seq_q, _ = q.shape
    attn = flash_attention(q, k, v, causal=causal, block_q=cfg.block_q, block_k=cfg.block_k)
    return attn.transpose(1, 2).reshape(batch, seq_q, cfg.dim) @ layer["wo"]


def init_kv_cache(cfg: ModelConfig, batch: int, cache_size: int, dtype=torch.float32,
                  device=None) -> Cache:
    """Zeroed fixed-size KV cache for every layer."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    shape = (batch, cfg.n_kv_heads, cache_size, cfg.head_dim)
    return [{"k": torch.zeros(shape, dtype=dtype, device=device),
             "v": torch.zeros(shape, dtype=dtype, device=device)} for _ in range(cfg.n_layers)]


def _cache_write(layer_cache: dict, k, v, start: int) -> dict:
    """Write ``k``/``v`` (length L) into slots ``(start + i) % C`` in place.

    With ``start + L <= C`` this is the reference's ``dynamic_update_slice`` at
    ``[start, start+L)`` (model.py:257-262); otherwise it wraps like the ring
    slots of model.py:437-449.
    """
    kc, vc = layer_cache["k"], layer_cache["v"]
    B, Hkv, C, D = kc.shape
    L = k.shape[2]
    kk = k.to(kc.dtype).contiguous()
    vv = v.to(vc.dtype).contiguous()
    _lib.check(_lib.lib().pf_cache_write(
        kc.data_ptr(), vc.data_ptr(), kk.data_ptr(), vv.data_ptr(), _lib.dtype_code(kc.dtype),
        B, Hkv, C, L, D, int(start), _lib.stream_of(kc)))
    return layer_cache


def prefill(params: Params, tokens, cfg: ModelConfig, interpret: bool = False,
            cache_size: Optional[int] = None):
    """Run the prompt and build the KV cache; returns ``(logits, cache)``."""
    batch, seq = tokens.shape
    if cache_size is None:
        cache_size = cfg.max_seq_len
    if cache_size < seq:
        raise ValueError(f"cache_size ({cache_size}) must be >= prompt length ({seq})")
    x = params["embed"][tokens]
    cos, sin = _rope_slice(0, seq, cfg, x.dtype, x.device)
    cache = init_kv_cache(cfg, batch, cache_size, x.dtype, x.device)
    mlp = None  # each block's MLP output is added by the next norm's launch
    for idx, layer in enumerate(params["layers"]):
        x, h = add_rms_norm(x, mlp, layer["attn_norm"], cfg.rms_norm_eps)
        q, k, v = project_qkv(layer, h, cfg)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        _cache_write(cache[idx], k, v, 0)
        x, h = add_rms_norm(x, _attend(layer, q, k, v, cfg, interpret, causal=True), layer["ffn_norm"],
                            cfg.rms_norm_eps)
        mlp = swiglu_mlp(h, layer["w_gate"], layer["w_up"], layer["w_down"])
    x, h = add_rms_norm(x, mlp, params["final_norm"], cfg.rms_norm_eps)
    return h @ params["lm_head"], cache


def _decode_layers(params: Params, token, cache: Cache, pos: int, slot: int, kv_len: int,
                   cfg: ModelConfig):
    x = params["embed"][token]
    cos, sin = _rope_slice(pos, 1, cfg, x.dtype, x.device)
    batch = x.shape[0]
    # The fixed (or ring) cache [B, Hkv, C, D] as a page pool of one C-token
    # page per sequence: RoPE of q/k and the k/v write at `slot` in one launch.
    table = torch.arange(batch, dtype=torch.int32, device=x.device).reshape(batch, 1)
    slots = torch.full((batch,), slot, dtype=torch.int32, device=x.device)
    rows = torch.zeros((batch,), dtype=torch.int32, device=x.device)
    if _fused_decode_ok(params, cfg, batch, x.dtype):
        # Projections with their norm / residual add / activation folded in:
        # 4 launches per block besides RoPE + cache write and attention.
        xw = x.reshape(batch, cfg.dim)  # the residual stream, updated in place
        eps = cfg.rms_norm_eps
        for layer, layer_cache in zip(params["layers"], cache):
            q = _qkv_rope_write(xw, layer, layer["attn_norm"], eps, cfg, layer_cache["k"], layer_cache["v"], cos, sin,
                                table, slots, rows)
            attn = flash_attention_decode(q, layer_cache["k"], layer_cache["v"], kv_len, block_k=cfg.block_k)
            _rows_linear(attn.reshape(batch, cfg.dim), _fused_rows(layer["wo"]), 1, residual=xw, out=xw)
            act = _rows_linear(xw, _fused_rows(layer["w_gate"], layer["w_up"]), 2, norm=layer["ffn_norm"], eps=eps)
            _rows_linear(act, _fused_rows(layer["w_down"]), 1, residual=xw, out=xw)
        # the final norm and lm_head (32000 columns) stay on the norm kernel + library matmul
        _, h = add_rms_norm(x, None, params["final_norm"], eps)
        return h @ params["lm_head"], cache
    mlp = None  # each block's MLP output is added by the next norm's launch
    for layer, layer_cache in zip(params["layers"], cache):
        x, h = add_rms_norm(x, mlp, layer["attn_norm"], cfg.rms_norm_eps)
        qkv = h @ _fused_columns(layer["wq"], layer["wk"], layer["wv"])  # one projection matmul
        q = rope_write_to_paged_cache_qkv(qkv, cfg.n_heads, layer_cache["k"], layer_cache["v"], cos, sin, table,
                                          slots, rows)
        attn = flash_attention_decode(q, layer_cache["k"], layer_cache["v"], kv_len,
                                      block_k=cfg.block_k)
        x, h = add_rms_norm(x, attn.transpose(1, 2).reshape(batch, 1, cfg.dim) @ layer["wo"],
                            layer["ffn_norm"], cfg.rms_norm_eps)
        mlp = swiglu_mlp(h, layer["w_gate"], layer["w_up"], layer["w_down"])
    x, h = add_rms_norm(x, mlp, params["final_norm"], cfg.rms_norm_eps)
    return h @ params["lm_head"], cache


def decode_step(params: Params, token, cache: Cache, pos: int, cfg: ModelConfig,
                interpret: bool = False):
    """Advance one token: write K/V at slot ``pos``, attend slots ``[0, pos]`` (model.py:307-356)."""
    cache_size = cache[0]["k"].shape[2]
    if pos >= cache_size:
        raise ValueError(f"position {pos} exceeds cache capacity {cache_size}")
    return _decode_layers(params, token, cache, pos, pos, pos + 1, cfg)


class DecodeGraph:
    """One decode step of every layer, captured once as a CUDA graph and replayed per token.

    A Python decode step issues ~100 small launches (8 layers of norms,
    projections, RoPE, cache write, attention, MLP); at batch 16 the host loop,
    not the GPU, sets the token rate.  Here the position lives on the device:
    the fixed (or ring) cache ``[B, Hkv, C, D]`` is addressed as a page pool of
    one ``C``-token page per sequence, RoPE and the cache write go through one
    fused kernel (table row ``pos``, slot ``pos % C``) and attention through the paged decode
    kernel with device lengths ``min(pos + 1, C)``, so one captured graph
    serves every position.  Kernels, split schedule and RoPE tables are those
    of ``decode_step`` / ``ring_decode_step``.
    """

    def __init__(self, params: Params, cache: Cache, cfg: ModelConfig, batch: int, dtype, device):
        self.params, self.cache, self.cfg = params, cache, cfg
        self.C = cache[0]["k"].shape[2]
        self.token = torch.zeros((batch, 1), dtype=torch.long, device=device)
        # the next step's input rows, written by the previous step's argmax + embedding kernel
        self.x = torch.zeros((batch, 1, cfg.dim), dtype=params["embed"].dtype, device=device)
        self.pos = torch.zeros((1,), dtype=torch.long, device=device)
        self.table = torch.arange(batch, dtype=torch.int32, device=device).reshape(batch, 1)
        self.slots = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.lens = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.rope_rows = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.dtype, self.device = dtype, device
        self.graph = None

    def _tables(self, last_pos: int):
        # rows are gathered from the table _rope_slice caches (same values, same dtype)
        self.cos, self.sin = _rope_slice(0, last_pos + 1, self.cfg, self.dtype, self.device)

    def _step(self):
        cfg, p = self.cfg, self.params
        # slot pos % C, live length min(pos + 1, C), RoPE row pos; then pos += 1
        _lib.check(_lib.lib().pf_decode_positions(self.pos.data_ptr(), self.C, self.slots.data_ptr(),
                                                  self.lens.data_ptr(), self.rope_rows.data_ptr(),
                                                  self.slots.numel(), _lib.stream_of(self.pos)))
        x = self.x
        batch = x.shape[0]
        if _fused_decode_ok(p, cfg, batch, x.dtype):
            # as _decode_layers: the residual stream is self.x, updated in place (the
            # argmax + embedding kernel writes the next step's rows over it at the end)
            xw = x.view(batch, cfg.dim)
            eps = cfg.rms_norm_eps
            for layer, lc in zip(p["layers"], self.cache):
                q = _qkv_rope_write(xw, layer, layer["attn_norm"], eps, cfg, lc["k"], lc["v"], self.cos, self.sin,
                                    self.table, self.slots, self.rope_rows)
                attn = paged_flash_attention(q, lc["k"], lc["v"], self.table, self.lens, max_context_len=self.C)
                _rows_linear(attn.reshape(batch, cfg.dim), _fused_rows(layer["wo"]), 1, residual=xw, out=xw)
                act = _rows_linear(xw, _fused_rows(layer["w_gate"], layer["w_up"]), 2, norm=layer["ffn_norm"],
                                   eps=eps)
                _rows_linear(act, _fused_rows(layer["w_down"]), 1, residual=xw, out=xw)
            _, h = add_rms_norm(x, None, p["final_norm"], eps)
            logits = (h @ p["lm_head"]).reshape(batch, -1)
        else:
            logits = self._step_unfused(x, batch)
        embed = p["embed"].contiguous()
        if embed.dtype != logits.dtype:
            raise ValueError("the embedding table and lm_head must share a dtype for the graph decode step")
        # greedy token (first maximum, as torch.argmax) and the next step's embedding row
        _lib.check(_lib.lib().pf_argmax_embed(logits.data_ptr(), logits.shape[-1], logits.shape[-1], batch,
                                              self.token.data_ptr(), embed.data_ptr(), self.x.data_ptr(),
                                              cfg.dim, _lib.dtype_code(logits.dtype), _lib.stream_of(logits)))

    def _step_unfused(self, x, batch):
        cfg, p = self.cfg, self.params
        mlp = None
        for layer, lc in zip(p["layers"], self.cache):
            x, h = add_rms_norm(x, mlp, layer["attn_norm"], cfg.rms_norm_eps)
            qkv = h @ _fused_columns(layer["wq"], layer["wk"], layer["wv"])
            q = rope_write_to_paged_cache_qkv(qkv, cfg.n_heads, lc["k"], lc["v"], self.cos, self.sin, self.table,
                                              self.slots, self.rope_rows)
            attn = paged_flash_attention(q, lc["k"], lc["v"], self.table, self.lens, max_context_len=self.C)
            x, h = add_rms_norm(x, attn.transpose(1, 2).reshape(batch, 1, cfg.dim) @ layer["wo"],
                                layer["ffn_norm"], cfg.rms_norm_eps)
            mlp = swiglu_mlp(h, layer["w_gate"], layer["w_up"], layer["w_down"])
        x, h = add_rms_norm(x, mlp, p["final_norm"], cfg.rms_norm_eps)
        return (h @ p["lm_head"]).reshape(batch, -1).contiguous()

    def capture(self, token, pos: int, last_pos: int):
        """One eager warm-up step at ``pos`` (it writes cache slot ``pos`` with the values the
        first replay writes there), then the capture of that step."""
        self._tables(last_pos)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._reset(token, pos)
            self._step()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self._reset(token, pos)

    def _reset(self, token, pos: int):
        self.token.copy_(token)
        self.pos.fill_(pos)
        self.x.copy_(self.params["embed"][self.token])

    def replay(self):
        self.graph.replay()
        return self.token


def _generate_graph(params: Params, prompt_ids, max_new_tokens: int, cfg: ModelConfig, logits, cache):
    batch, prompt_len = prompt_ids.shape
    next_tok = _argmax_last(logits).to(prompt_ids.dtype)
    out = torch.empty((batch, prompt_len + max_new_tokens), dtype=prompt_ids.dtype, device=prompt_ids.device)
    out[:, :prompt_len] = prompt_ids
    out[:, prompt_len:prompt_len + 1] = next_tok
    if max_new_tokens > 1:
        g = DecodeGraph(params, cache, cfg, batch, params["embed"].dtype, prompt_ids.device)
        g.capture(next_tok, prompt_len, prompt_len + max_new_tokens)
        for i in range(max_new_tokens - 1):
            out[:, prompt_len + 1 + i:prompt_len + 2 + i] = g.replay()
    return out


def generate_cached(params: Params, prompt_ids, max_new_tokens: int, cfg: ModelConfig,
                    interpret: bool = False, cache_size: Optional[int] = None, use_graph: bool = True):
    """Greedy generation with a fixed-size KV cache (model.py:359-386).

    ``cache_size`` defaults to ``prompt_len + max_new_tokens`` as in the
    reference; a larger capacity (e.g. 512) may be given.  With ``use_graph``
    (default) the decode steps replay one captured CUDA graph (``DecodeGraph``).
    """
    batch, prompt_len = prompt_ids.shape
    if cache_size is None:
        cache_size = prompt_len + max_new_tokens
    logits, cache = prefill(params, prompt_ids, cfg, cache_size=cache_size)
    if use_graph:
        if prompt_len + max_new_tokens - 1 > cache_size:
            raise ValueError(f"position {prompt_len + max_new_tokens - 2} exceeds cache capacity {cache_size}")
        return _generate_graph(params, prompt_ids, max_new_tokens, cfg, logits, cache)
    next_tok = _argmax_last(logits).to(prompt_ids.dtype)
    out = [prompt_ids, next_tok]
    for i in range(max_new_tokens - 1):
        logits, cache = decode_step(params, next_tok, cache, prompt_len + i, cfg)
        next_tok = _argmax_last(logits).to(prompt_ids.dtype)
        out.append(next_tok)
    return torch.cat(out, dim=1)


# --------------------------------------------------------------------------- #
# Ring-buffer cache (model.py:389-531)
# --------------------------------------------------------------------------- #
def init_ring_cache(cfg: ModelConfig, batch: int, capacity: int, dtype=torch.float32,
                    device=None) -> Cache:
    """Ring-buffer KV cache holding the most recent ``capacity`` tokens."""
    return init_kv_cache(cfg, batch, capacity, dtype, device)


def ring_kv_len(total_tokens: int, capacity: int) -> int:
    """Number of live slots after ``total_tokens`` have been written."""
    return min(total_tokens, capacity)


def prefill_ring(params: Params, tokens, cfg: ModelConfig, capacity: int,
                 interpret: bool = False):
    """Prefill into a ring cache keeping the last ``capacity`` tokens at slots ``pos % capacity``."""
    batch, seq = tokens.shape
    x = params["embed"][tokens]
    cos, sin = _rope_slice(0, seq, cfg, x.dtype, x.device)
    keep = min(seq, capacity)
    start = seq - keep
    cache = init_ring_cache(cfg, batch, capacity, x.dtype, x.device)
    mlp = None  # each block's MLP output is added by the next norm's launch
    for idx, layer in enumerate(params["layers"]):
        x, h = add_rms_norm(x, mlp, layer["attn_norm"], cfg.rms_norm_eps)
        q, k, v = project_qkv(layer, h, cfg)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        _cache_write(cache[idx], k[:, :, start:], v[:, :, start:], start)
        x, h = add_rms_norm(x, _attend(layer, q, k, v, cfg, interpret, causal=True), layer["ffn_norm"],
                            cfg.rms_norm_eps)
        mlp = swiglu_mlp(h, layer["w_gate"], layer["w_up"], layer["w_down"])
    x, h = add_rms_norm(x, mlp, params["final_norm"], cfg.rms_norm_eps)
    return h @ params["lm_head"], cache


def ring_decode_step(params: Params, token, cache: Cache, pos: int, cfg: ModelConfig,
                     interpret: bool = False):
    """One decode step against a ring cache: write slot ``pos % C``, attend the live window."""
    capacity = cache[0]["k"].shape[2]
    return _decode_layers(params, token, cache, pos, pos % capacity,
                          ring_kv_len(pos + 1, capacity), cfg)


def generate_streaming(params: Params, prompt_ids, max_new_tokens: int, cfg: ModelConfig,
                       window: int, interpret: bool = False, use_graph: bool = True):
    """Greedy generation in constant memory with a ring-buffer cache of ``window`` slots.

    With ``use_graph`` (default) the decode steps replay one captured CUDA graph
    whose slot ``pos % window`` and live length ``min(pos + 1, window)`` are
    computed on the device.
    """
    batch, prompt_len = prompt_ids.shape
    logits, cache = prefill_ring(params, prompt_ids, cfg, window)
    if use_graph:
        return _generate_graph(params, prompt_ids, max_new_tokens, cfg, logits, cache)
    next_tok = _argmax_last(logits).to(prompt_ids.dtype)
    out: List[torch.Tensor] = [prompt_ids, next_tok]
    for i in range(max_new_tokens - 1):
        logits, cache = ring_decode_step(params, next_tok, cache, prompt_len + i, cfg)
        next_tok = _argmax_last(logits).to(prompt_ids.dtype)
        out.append(next_tok)
    return torch.cat(out, dim=1)
