"""The attention-backend seam of PagedServe, restated for standalone use.

These are the reference's interface types (pagedserve/attention/backend.py:44-193)
with the same names, fields, properties and method signatures, so that
``PagedCudaBackend`` is a drop-in: an engine written against the reference's
``AttentionBackend`` calls it exactly as it calls ``ContiguousAttentionBackend``,
and objects of the reference's own ``StepInput`` class are accepted as-is
(only attributes are read). They are restated, not imported, because the
backend must run where the reference is not installed.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any

import torch

__all__ = ["AttentionBackend", "AttentionMetadata", "KVMemoryStats", "StepInput"]


@dataclass(frozen=True)
class KVMemoryStats:
    """Reserved KV bytes versus KV bytes holding real tokens (backend.py:44-79)."""

    allocated_bytes: int
    live_bytes: int

    @property
    def utilization(self) -> float | None:
        """live / allocated, or None when nothing is allocated."""
        if self.allocated_bytes <= 0:
            return None
        return self.live_bytes / self.allocated_bytes

    @property
    def wasted_bytes(self) -> int:
        return max(0, self.allocated_bytes - self.live_bytes)

    def to_dict(self) -> dict[str, Any]:
        return {
            "allocated_bytes": self.allocated_bytes,
            "live_bytes": self.live_bytes,
            "wasted_bytes": self.wasted_bytes,
            "utilization": self.utilization,
        }


@dataclass(frozen=True)
class StepInput:
    """One forward pass, described independently of KV layout (backend.py:82-122).

    Attributes:
        query_len: tokens per sequence in this step (1 for decode).
        context_len: tokens cached per sequence before this step (shared index
            under left padding).
        seq_lens: [num_seqs] real tokens per sequence after this step.
        padding_mask: [num_seqs, context_len + query_len], True on real tokens.
        is_prefill: whether this step processes prompts.
        block_tables: [num_seqs, max_blocks] int32 physical block ids, or None
            for a backend-managed identity layout.
        slot_mapping: [num_seqs * query_len] int64 flat slots of this step's
            tokens (-1 = padding), or None.
    """

    query_len: int
    context_len: int
    seq_lens: torch.Tensor
    padding_mask: torch.Tensor
    is_prefill: bool
    block_tables: torch.Tensor | None = None
    slot_mapping: torch.Tensor | None = None

    @property
    def num_seqs(self) -> int:
        return int(self.padding_mask.shape[0])

    @property
    def key_len(self) -> int:
        return self.context_len + self.query_len


class AttentionMetadata:
    """Backend-private per-step state, built once per step and reused by every layer."""


class AttentionBackend(ABC):
    """How KV is stored, written and read (backend.py:138-193)."""

    name: str = "abstract"

    @abstractmethod
    def allocate(self, num_seq_slots: int, max_seq_len: int) -> None:
        """Reserve KV storage up front (never in the decode loop)."""

    @abstractmethod
    def free(self) -> None:
        """Release KV storage. Safe to call when nothing is allocated."""

    @abstractmethod
    def begin_step(self, step: StepInput) -> AttentionMetadata:
        """Prepare per-step state before any layer runs."""

    @abstractmethod
    def forward(
        self,
        layer_idx: int,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        metadata: AttentionMetadata,
    ) -> torch.Tensor:
        """Write this step's K/V into the cache and attend over everything cached.

        query [num_seqs, query_len, Hq, D]; key/value [num_seqs, query_len, Hkv, D]
        (RoPE applied); returns [num_seqs, query_len, Hq, D].
        """

    @abstractmethod
    def memory_stats(self) -> KVMemoryStats:
        """Reserved versus live KV bytes, as of the last completed step."""
