"""Generates tests/golden/attention_cases.npz -- fixtures that pin the CPU oracle.

The reference (JAX/Pallas) cannot run in this environment (no jax), and its
tests store no vectors.  These fixtures are computed by an implementation
independent of oracle/attention_oracle.py: float64 PyTorch autograd through the
reference's naive attention (src/pallas_flash/reference.py:45-66: GQA head
repetition, causal -1e30 mask, softmax, weights @ v) -- the same quantity the
reference's tests compare its kernels with (tests/test_flash_attention.py:33-41,
tests/test_backward.py:107-119).  Inputs are seeded N(0, 1) (numpy
default_rng), stored in float32.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).with_name("attention_cases.npz")

# (name, B, H, Hkv, Sq, Sk, D, causal, kv_len, sm_scale)
CASES = [
    ("mha_noncausal", 1, 2, 2, 40, 40, 16, False, None, None),
    ("mha_causal_ragged", 1, 2, 2, 37, 37, 16, True, None, None),
    ("gqa_causal", 2, 4, 2, 33, 33, 8, True, None, None),
    ("mqa_noncausal", 1, 4, 1, 24, 24, 8, False, None, None),
    ("kvlen_decode", 1, 4, 2, 1, 48, 16, False, 19, None),
    ("custom_scale", 1, 2, 2, 20, 20, 16, False, None, 0.05),
    ("cross_causal", 1, 2, 1, 12, 30, 8, True, None, None),
]


def torch_reference(q, k, v, causal, sm_scale, kv_len):
    if kv_len is not None:
        k, v = k[:, :, :kv_len], v[:, :, :kv_len]
    H, Hkv = q.shape[1], k.shape[1]
    if H != Hkv:
        k = k.repeat_interleave(H // Hkv, dim=1)
        v = v.repeat_interleave(H // Hkv, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * sm_scale
    if causal:
        qp = torch.arange(q.shape[2])[:, None]
        kp = torch.arange(k.shape[2])[None, :]
        s = torch.where(qp >= kp, s, torch.full_like(s, -1e30))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, dim=-1), v)


def main() -> None:
    rng = np.random.default_rng(20260101)
    arrays = {}
    for name, B, H, Hkv, Sq, Sk, D, causal, kv_len, scale in CASES:
        q = rng.standard_normal((B, H, Sq, D)).astype(np.float32)
        k = rng.standard_normal((B, Hkv, Sk, D)).astype(np.float32)
        v = rng.standard_normal((B, Hkv, Sk, D)).astype(np.float32)
        do = rng.standard_normal((B, H, Sq, D)).astype(np.float32)
        sm = scale if scale is not None else 1.0 / np.sqrt(D)
        tq, tk, tv = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v))
        out = torch_reference(tq, tk, tv, causal, sm, kv_len)
        (out * torch.tensor(do, dtype=torch.float64)).sum().backward()
        meta = np.array([B, H, Hkv, Sq, Sk, D, int(causal), -1 if kv_len is None else kv_len],
                        dtype=np.int64)
        arrays.update({
            f"{name}/meta": meta, f"{name}/scale": np.array(sm, dtype=np.float64),
            f"{name}/q": q, f"{name}/k": k, f"{name}/v": v, f"{name}/do": do,
            f"{name}/out": out.detach().numpy(), f"{name}/dq": tq.grad.numpy(),
            f"{name}/dk": tk.grad.numpy(), f"{name}/dv": tv.grad.numpy(),
        })
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
