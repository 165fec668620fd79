"""Geometry the paged backend reads from its configuration objects.

``PagedCudaBackend`` reads only the attributes below, so the reference's own
``ModelConfig`` and ``CacheConfig`` (pagedserve/config.py:61-213) can be passed
unchanged; these dataclasses carry the same field names for standalone use.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["CacheConfig", "ModelConfig"]


@dataclass(frozen=True)
class ModelConfig:
    """Attention geometry (the subset of pagedserve/config.py:61-108 this path uses)."""

    name: str
    num_layers: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float = 10000.0
    max_position_embeddings: int = 2048

    def __post_init__(self) -> None:
        if self.num_q_heads % self.num_kv_heads != 0:
            raise ValueError(
                f"num_q_heads ({self.num_q_heads}) must be divisible by "
                f"num_kv_heads ({self.num_kv_heads}); GQA groups would be ragged"
            )

    @property
    def num_queries_per_kv(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    def kv_bytes_per_token(self, dtype: torch.dtype) -> int:
        """KV bytes one token occupies over all layers: K and V, every KV head
        (pagedserve/config.py:99-108)."""
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * (
            torch.finfo(dtype).bits // 8)


@dataclass(frozen=True)
class CacheConfig:
    """KV cache sizing (pagedserve/config.py:186-213); ``block_size`` is the page size."""

    max_seq_len: int = 2048
    max_num_seqs: int = 32
    block_size: int = 16
    gpu_memory_utilization: float = 0.90
