"""Seeded workload generators: shapes, disjoint block assignment, LPT sharding."""

from __future__ import annotations

import math

import pytest
import torch

from paged_serve_b200.workloads import (
    SPECS,
    append_workload,
    decode_workload,
    lpt_shard,
    prefix_workload,
)


def _blocks_used(wl):
    bs = wl.spec.block_size
    ids = []
    for i, n in enumerate(wl.ctx_lens.tolist()):
        ids.extend(wl.block_tables[i, : (n + bs - 1) // bs].tolist())
    return ids


def test_llama8b_shape_and_pool():
    wl = decode_workload("llama8b", seed=0)
    assert wl.batch == 256
    assert int(wl.ctx_lens.min()) >= 512 and int(wl.ctx_lens.max()) <= 4096
    ids = _blocks_used(wl)
    assert len(ids) == len(set(ids)), "sequences must not share blocks"
    assert max(ids) < wl.num_blocks
    assert wl.num_blocks == math.ceil(1.25 * len(ids))
    assert wl.block_tables.shape[1] == 4096 // 16
    # algorithmic bytes per layer ~ 2.4-2.6 GB for this draw (K+V dominate)
    assert 2.0e9 < wl.algorithmic_bytes_per_layer() < 3.0e9


def test_tiny_matches_plumbing_workload():
    wl = decode_workload("tiny", seed=0)
    assert wl.ctx_lens.tolist() == [17, 64, 100, 255]
    assert wl.num_blocks == 128
    ids = _blocks_used(wl)
    assert len(set(ids)) == len(ids) == 2 + 4 + 7 + 16


def test_seeded_draws_are_reproducible():
    a = decode_workload("llama8b", seed=3)
    b = decode_workload("llama8b", seed=3)
    assert torch.equal(a.ctx_lens, b.ctx_lens) and torch.equal(a.block_tables, b.block_tables)


def test_lpt_balances_tokens_and_covers_everything():
    lens = torch.randint(128, 32768, (512,), generator=torch.Generator().manual_seed(1))
    for world in (1, 2, 4, 8):
        shards = lpt_shard(lens, world)
        allidx = torch.cat(shards).sort().values
        assert torch.equal(allidx, torch.arange(512))
        loads = [int(lens[s].sum()) for s in shards]
        # LPT bound: max load <= mean + the longest job
        assert max(loads) <= sum(loads) / world + int(lens.max())


def test_weak_scaled_shards_partition_the_global_batch():
    world = 4
    seen = []
    for r in range(world):
        wl = decode_workload("llama8b", seed=0, rank=r, world=world)
        seen.extend(wl.seq_ids.tolist())
        ids = _blocks_used(wl)
        assert len(ids) == len(set(ids)) and max(ids) < wl.num_blocks
    assert sorted(seen) == list(range(256 * world))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_weak_scaling_gives_every_rank_the_one_gpu_lengths(world):
    """Per-GPU work is fixed as the world grows: each rank's share of the weak
    global batch is the one-GPU draw's multiset of lengths."""
    one = sorted(decode_workload("llama8b", seed=0).ctx_lens.tolist())
    for r in range(world):
        wl = decode_workload("llama8b", seed=0, rank=r, world=world)
        assert sorted(wl.ctx_lens.tolist()) == one


def test_strong_scaling_splits_one_batch():
    whole = decode_workload("llama70b", seed=0, weak=False)
    parts = [decode_workload("llama70b", seed=0, rank=r, world=4, weak=False) for r in range(4)]
    assert sum(p.batch for p in parts) == whole.batch == 512
    assert sorted(x for p in parts for x in p.ctx_lens.tolist()) == sorted(whole.ctx_lens.tolist())
    loads = [p.total_tokens for p in parts]
    assert max(loads) / (sum(loads) / 4) < 1.001


def test_llama70b_lognormal_clipped():
    wl = decode_workload("llama70b", seed=0)
    assert SPECS["llama70b"].sigma == 1.0
    assert wl.batch == 512
    assert int(wl.ctx_lens.min()) >= 128 and int(wl.ctx_lens.max()) <= 32768
    med = float(wl.ctx_lens.float().median())
    assert 1500 < med < 2800


def test_append_workload_slots_unique_and_positions():
    wl = append_workload(seed=0)
    assert wl.num_tokens == 256 + 8 * 2048
    assert wl.slot_mapping.unique().numel() == wl.num_tokens
    assert int(wl.slot_mapping.max()) < wl.num_blocks * 16
    assert wl.positions[256:2304].tolist() == list(range(2048))


def test_prefix_workload_shares_and_forks():
    wl = prefix_workload(seed=0)
    assert wl.batch == 64 and wl.total_q == 64 * 512
    assert wl.cow_pairs.shape == (8, 2)
    shared = set(wl.shared_blocks.tolist())
    # forking sequences reference their private copy, not the shared block
    for i in range(56, 64):
        assert int(wl.prefix_lens[i]) == 1000
        assert int(wl.block_tables[i, 62]) not in shared
        assert int(wl.block_tables[i, 62]) == int(wl.cow_pairs[i - 56, 1])
    for i in range(56):
        assert wl.block_tables[i, :64].tolist() == wl.shared_blocks.tolist()
    # new tokens of distinct sequences never share a slot
    assert wl.slot_mapping.unique().numel() == wl.total_q
    # 686 GFLOP of causal pairs on one layer
    assert abs(wl.causal_flops() / 1e9 - 686) < 10
