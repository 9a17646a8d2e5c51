"""pallas_flash for NVIDIA B200 (sm_100a).

The public API of the JAX/Pallas ``pallas_flash`` package (FlashAttention
forward/backward with saved log-sum-exp, fixed-cache decode, fused RoPE, paged
decode, and the tiny-LLaMA generation paths), with every attention kernel a
hand-written sm_100a CUDA kernel in ``libpallas_flash_b200.so`` reached through
its C ABI.  Operands are CUDA ``torch.Tensor``s.
"""

from .config import ModelConfig
from .flash_attention import (
    flash_attention,
    flash_attention_backward,
    flash_attention_decode,
    flash_attention_with_lse,
)
from .fused_rope import flash_attention_rope, rope_apply
from .paged import (
    gather_paged,
    init_paged_cache,
    paged_flash_attention,
    paged_prefill_attention,
    write_to_paged_cache,
    write_to_paged_cache_batch,
    rope_write_to_paged_cache_batch,
    rope_write_to_paged_cache_qkv,
)
from .reference import reference_attention
from .model import (
    forward,
    generate,
    generate_cached,
    prefill,
    decode_step,
    init_kv_cache,
    init_ring_cache,
    ring_kv_len,
    prefill_ring,
    ring_decode_step,
    generate_streaming,
    init_params,
    decoder_block,
    project_qkv,
    rms_norm,
    apply_rope,
    precompute_rope,
    swiglu_mlp,
    add_rms_norm,
    silu_mul,
)

__all__ = [
    "ModelConfig",
    "flash_attention",
    "flash_attention_decode",
    "flash_attention_rope",
    "rope_apply",
    "paged_flash_attention",
    "paged_prefill_attention",
    "init_paged_cache",
    "write_to_paged_cache",
    "reference_attention",
    "forward",
    "generate",
    "generate_cached",
    "prefill",
    "decode_step",
    "init_kv_cache",
    "init_ring_cache",
    "ring_kv_len",
    "prefill_ring",
    "ring_decode_step",
    "generate_streaming",
    "init_params",
    "decoder_block",
    "project_qkv",
    "rms_norm",
    "apply_rope",
    "precompute_rope",
    "swiglu_mlp",
    # additions of this build
    "add_rms_norm",
    "silu_mul",
    "flash_attention_with_lse",
    "flash_attention_backward",
    "write_to_paged_cache_batch",
    "rope_write_to_paged_cache_batch",
    "rope_write_to_paged_cache_qkv",
    "gather_paged",
]

__version__ = "0.1.0"
