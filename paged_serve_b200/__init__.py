"""paged_serve_b200 — B200-native (sm_100a) KV-memory hot path of PagedServe.

Hand-written CUDA kernels behind a C ABI (``include/paged_serve.h``) for the
four operations of the reference's attention seam: paged decode attention,
KV append (optionally with RoPE fused on K), block copy, and causal paged
prefill; plus ``PagedCudaBackend``, a drop-in ``AttentionBackend``.
"""

from paged_serve_b200.config import CacheConfig, ModelConfig
from paged_serve_b200.interface import AttentionBackend, AttentionMetadata, KVMemoryStats, StepInput

__all__ = [
    "AttentionBackend",
    "AttentionMetadata",
    "CacheConfig",
    "KVMemoryStats",
    "ModelConfig",
    "PagedCudaBackend",
    "StepInput",
]


def __getattr__(name):
    if name == "PagedCudaBackend":
        from paged_serve_b200.backend import PagedCudaBackend

        return PagedCudaBackend
    raise AttributeError(name)
