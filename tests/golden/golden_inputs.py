"""Deterministic inputs for the reference-generated golden vectors.

The golden file stores only outputs; both the generator
(``make_reference_golden.py``) and the tests rebuild the inputs from
``(shape, seed)`` with this counter-based generator, which depends on no
library's random stream: SplitMix64 over the element index, two 32-bit
uniforms per element, Box-Muller to N(0, 1), then round-to-nearest-even to
bfloat16 (returned as float32), so the same inputs serve fp32 and bf16 tests.
"""

from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLD
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def randn(shape, seed: int) -> np.ndarray:
    """Seeded N(0, 1) values, bfloat16-representable, as float32."""
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.uint64) + (np.uint64(seed) << np.uint64(40))
    r = _splitmix64(idx)
    u1 = ((r >> np.uint64(40)).astype(np.float64) + 0.5) / float(1 << 24)
    u2 = ((r & np.uint64(0xFFFFFF)).astype(np.float64)) / float(1 << 24)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return bf16_round(z.astype(np.float32).reshape(shape))


def randint(shape, high: int, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.uint64) + (np.uint64(seed) << np.uint64(40))
    return (_splitmix64(idx) % np.uint64(high)).astype(np.int64).reshape(shape)


def permutation(n: int, seed: int) -> np.ndarray:
    """A seeded permutation of range(n) (argsort of hashed keys)."""
    keys = _splitmix64(np.arange(n, dtype=np.uint64) + (np.uint64(seed) << np.uint64(40)))
    return np.argsort(keys, kind="stable").astype(np.int64)


# Inputs of each golden group, shared by the generator and the tests.
FWD_CASES = [  # (name, B, H, Hkv, Sq, Sk, D, causal, kv_len, bq, bk, seed)
    ("s128", 1, 1, 1, 128, 128, 128, True, None, 128, 128, 1),
    ("s256_mha", 1, 2, 2, 256, 256, 128, False, None, 128, 128, 2),
    ("s384_b2", 2, 2, 2, 384, 384, 64, True, None, 128, 128, 3),
    ("s200_ragged", 1, 2, 2, 200, 200, 128, True, None, 128, 128, 4),
    ("s130_ragged", 1, 2, 2, 130, 130, 128, False, None, 128, 128, 5),
    ("gqa8x2_causal", 1, 8, 2, 256, 256, 64, True, None, 128, 128, 6),
    ("mqa8x1", 1, 8, 1, 256, 256, 64, False, None, 128, 128, 7),
    ("blk64", 1, 2, 2, 384, 384, 64, True, None, 64, 64, 8),
    ("blk128x256", 1, 2, 2, 384, 384, 64, True, None, 128, 256, 8),
    ("blk256x128", 1, 2, 2, 384, 384, 64, True, None, 256, 128, 8),
    ("kvlen_cross", 2, 4, 2, 64, 320, 64, False, 201, 128, 128, 9),
    ("kvlen_causal", 1, 4, 2, 192, 192, 64, True, 150, 128, 128, 10),
    ("config1", 1, 8, 8, 512, 512, 128, True, None, 128, 128, 11),
]

BWD_CASES = [  # (name, B, H, Hkv, S, D, causal, bq, bk, seed)
    ("s128_causal", 1, 2, 2, 128, 128, True, 128, 128, 21),
    ("s256_noncausal", 1, 2, 2, 256, 64, False, 128, 128, 22),
    ("b2_s256_causal", 2, 2, 2, 256, 64, True, 128, 128, 23),
    ("gqa_s256_causal", 1, 4, 2, 256, 64, True, 128, 128, 24),
    ("mqa_s256_noncausal", 1, 4, 1, 256, 64, False, 128, 128, 25),
    ("s200_ragged_causal", 1, 2, 2, 200, 128, True, 128, 128, 26),
    ("blk64_causal", 1, 2, 2, 256, 64, True, 64, 64, 27),
]

DEC_KV = (4, 2, 1)
DEC_LENS = (1, 5, 130, 256)

ROPE_CASES = [  # (name, B, H, Hkv, S, causal, seed)
    ("h2kv2_causal", 1, 2, 2, 256, True, 41), ("h4kv2_noncausal", 1, 4, 2, 256, False, 42),
    ("h4kv1_causal", 1, 4, 1, 256, True, 43), ("ragged130", 2, 2, 2, 130, True, 44),
    ("ragged200", 1, 2, 2, 200, True, 45),
]

PAGED_CASES = [  # test_paged.py:31-38: (B, H, Hkv, page_size, context_lens)
    (1, 2, 2, 64, [100]), (3, 4, 2, 64, [10, 130, 200]),
    (2, 4, 1, 128, [128, 5]), (4, 2, 2, 32, [1, 33, 64, 90]),
]

MODEL_CASES = [  # (name, n_heads, n_kv, head_dim, ffn, n_layers, prompt, n_new, window, seed)
    ("mha_d128", 2, 2, 128, 512, 2, [[3, 1, 4, 1, 5], [2, 7, 1, 8, 2]], 12, 8, 61),
    ("gqa_d64", 4, 2, 64, 384, 3, [[5, 9, 2, 7, 1, 6, 6, 3]], 16, 6, 62),
]


def fwd_inputs(case):
    name, B, H, Hkv, Sq, Sk, D, causal, kv_len, bq, bk, seed = case
    return (randn((B, H, Sq, D), seed * 8 + 1), randn((B, Hkv, Sk, D), seed * 8 + 2),
            randn((B, Hkv, Sk, D), seed * 8 + 3))


def bwd_inputs(case):
    name, B, H, Hkv, S, D, causal, bq, bk, seed = case
    return (randn((B, H, S, D), seed * 8 + 1), randn((B, Hkv, S, D), seed * 8 + 2),
            randn((B, Hkv, S, D), seed * 8 + 3), randn((B, H, S, D), seed * 8 + 4))


def dec_inputs(n_kv):
    return (randn((1, 4, 1, 128), 300 + n_kv), randn((1, n_kv, 256, 128), 310 + n_kv),
            randn((1, n_kv, 256, 128), 320 + n_kv))


def rope_inputs(case):
    name, B, H, Hkv, S, causal, seed = case
    return (randn((B, H, S, 128), seed * 8 + 1), randn((B, Hkv, S, 128), seed * 8 + 2),
            randn((B, Hkv, S, 128), seed * 8 + 3))


def rope_decode_inputs():
    return randn((1, 2, 1, 128), 501), randn((1, 2, 128, 128), 502), randn((1, 2, 128, 128), 503)


def paged_inputs(i):
    B, H, Hkv, ps, lens = PAGED_CASES[i]
    num_pages, D = 32, 128
    return (randn((B, H, 1, D), 600 + i), randn((num_pages, Hkv, ps, D), 610 + i),
            randn((num_pages, Hkv, ps, D), 620 + i))


def paged_write_inputs():
    return randn((1, 2, 70, 128), 650), randn((1, 2, 70, 128), 651), randn((1, 2, 1, 128), 652)


def model_params(case):
    """Parameters with init_params' shapes and scales (model.py:146-176), bf16-valued."""
    name, H, Hkv, hd, ffn, nl, prompt, n_new, window, seed = case
    dim, kv_dim, vocab = H * hd, Hkv * hd, 64
    ctr = [seed * 1000]

    def normal(shape, scale):
        ctr[0] += 1
        return bf16_round(randn(shape, ctr[0]) * np.float32(scale))

    proj = 1.0 / dim ** 0.5
    params = {"embed": normal((vocab, dim), 0.02), "layers": []}
    for _ in range(nl):
        params["layers"].append({
            "attn_norm": np.ones((dim,), np.float32), "ffn_norm": np.ones((dim,), np.float32),
            "wq": normal((dim, dim), proj), "wk": normal((dim, kv_dim), proj),
            "wv": normal((dim, kv_dim), proj), "wo": normal((dim, dim), proj),
            "w_gate": normal((dim, ffn), proj), "w_up": normal((dim, ffn), proj),
            "w_down": normal((ffn, dim), 1.0 / ffn ** 0.5),
        })
    params["final_norm"] = np.ones((dim,), np.float32)
    params["lm_head"] = normal((dim, vocab), proj)
    return params
