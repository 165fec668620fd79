"""Shared pytest configuration.

Marker ``gpu``: needs a CUDA device (a B200) and the built native library.
``python -m pytest tests -m "not gpu"`` runs everything else on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA GPU (B200) and the native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def pool_from_sequences(flat: torch.Tensor, lens: list[int], tables: torch.Tensor,
                        num_blocks: int, block_size: int) -> torch.Tensor:
    """Scatter concatenated per-sequence rows [sum(lens), Hkv, D] into a zeroed pool."""
    hkv, d = flat.shape[1:]
    pool = torch.zeros((num_blocks, hkv, block_size, d), dtype=flat.dtype)
    start = 0
    for i, n in enumerate(lens):
        seq = flat[start : start + n]
        start += n
        for j in range((n + block_size - 1) // block_size):
            chunk = seq[j * block_size : (j + 1) * block_size]
            pool[int(tables[i, j]), :, : chunk.shape[0]] = chunk.transpose(0, 1)
    return pool


@pytest.fixture(scope="session")
def golden():
    return load_golden
