"""Naive attention, the baseline op of the public API (src/pallas_flash/reference.py:22-66).

``reference_attention`` materialises the full ``[Sq, Sk]`` score matrix with
plain PyTorch ops on whatever device its inputs live on -- the B200 analogue
of the reference's XLA baseline, kept because the reference exports it.  It is
not used by any kernel path; the parity oracle used by the tests is the
separate CPU restatement under ``oracle/``.
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def reference_attention(q, k, v, *, causal: bool = False, sm_scale: Optional[float] = None):
    """Standard scaled dot-product attention with GQA head repetition.

    Scores are formed in the input dtype, up-cast to fp32 and scaled; the causal
    mask uses -1e30; softmax and ``weights @ v`` run in fp32; the result is cast
    back to ``q.dtype`` -- step for step the reference's computation.
    """
    head_dim = q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    num_heads, num_kv_heads = q.shape[1], k.shape[1]
    if num_kv_heads != num_heads:
        rep = num_heads // num_kv_heads
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    scores = torch.einsum("bhqd,bhkd->bhqk", q, k).to(torch.float32) * sm_scale
    if causal:
        sq, sk = q.shape[2], k.shape[2]
        qp = torch.arange(sq, device=q.device)[:, None]
        kp = torch.arange(sk, device=q.device)[None, :]
        scores = torch.where(qp >= kp, scores, torch.full_like(scores, -1e30))
    weights = torch.softmax(scores, dim=-1)
    out = torch.einsum("bhqk,bhkd->bhqd", weights, v.to(torch.float32))
    return out.to(q.dtype)
