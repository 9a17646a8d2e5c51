"""Configuration for the tiny LLaMA model (behaviour of src/pallas_flash/config.py:8-55)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModelConfig:
    """Hyper-parameters of the tiny LLaMA decoder.

    Same fields, defaults and validation as the reference: ``n_kv_heads == 0``
    means plain multi-head attention (it becomes ``n_heads``), ``dim`` must be
    ``n_heads * head_dim`` and ``n_heads`` a multiple of ``n_kv_heads``.
    ``block_q``/``block_k`` are kept for API compatibility (the B200 kernels
    pick their own tiles).
    """

    vocab_size: int = 256
    dim: int = 256
    n_layers: int = 4
    n_heads: int = 2
    n_kv_heads: int = 0
    head_dim: int = 128
    ffn_hidden: int = 688
    max_seq_len: int = 512
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    block_q: int = 128
    block_k: int = 128

    def __post_init__(self) -> None:
        if self.n_kv_heads == 0:
            object.__setattr__(self, "n_kv_heads", self.n_heads)
        if self.dim != self.n_heads * self.head_dim:
            raise ValueError(
                f"dim ({self.dim}) must equal n_heads * head_dim "
                f"({self.n_heads} * {self.head_dim} = {self.n_heads * self.head_dim})"
            )
        if self.n_kv_heads <= 0 or self.n_heads % self.n_kv_heads != 0:
            raise ValueError(
                f"n_heads ({self.n_heads}) must be a multiple of n_kv_heads "
                f"({self.n_kv_heads})"
            )

    @property
    def kv_dim(self) -> int:
        """Total width of the key/value projections."""
        return self.n_kv_heads * self.head_dim
