"""RoPE cos/sin table for the fused append (built once per backend, not per step)."""

from __future__ import annotations

import torch

__all__ = ["cos_sin_table"]


def cos_sin_table(
    head_dim: int,
    theta: float,
    max_positions: int,
    dtype: torch.dtype,
    device: torch.device | str,
) -> torch.Tensor:
    """``[max_positions, head_dim]`` table whose row p is cos half | sin half.

    Computed with the same torch ops, on the same device, as the reference's
    ``RotaryEmbedding`` (pagedserve/model/layers.py:91-116): fp32
    ``inv_freq = 1/theta**(arange(0, D, 2)/D)``, fp32 angles ``pos*inv_freq``,
    ``cos``/``sin`` in fp32, then one cast to ``dtype``. Because the reference's
    ``emb = cat(freqs, freqs)`` repeats the angles, its cos/sin rows are this
    table's halves repeated, so the kernel reads half as many bytes and the
    rotated K is bit-identical to ``apply_rotary`` run on this device.
    """
    if head_dim % 2:
        raise ValueError("head_dim must be even for rotary embeddings")
    device = torch.device(device)
    inv_freq = 1.0 / (
        theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim)
    )
    pos = torch.arange(max_positions, device=device)
    freqs = pos.float().unsqueeze(-1) * inv_freq.view(1, -1)
    return torch.cat((freqs.cos().to(dtype), freqs.sin().to(dtype)), dim=-1).contiguous()
