"""Block manager and prefix cache (host logic, CPU).

The reference lists the manager's contract (AGENTS.md:127-129: free list, block
tables, refcounts, alloc/free/fork, hash-chain prefix cache with an LRU
evictor) and its debug invariants (AGENTS.md:229-238) without code; these tests
hold :class:`BlockManager` to that contract. The slots a plan implies are
checked here with :meth:`StepPlan.slot`; the device builder that produces them
is compared with the same formula in ``test_gpu_block_manager.py``.
"""

from __future__ import annotations

import random

import pytest

from paged_serve_b200.block_manager import BlockManager, NoFreeBlocksError

BS = 16


def _mgr(n=64, cache=False):
    return BlockManager(n, BS, enable_prefix_caching=cache, debug_invariants=True)


def test_allocate_free_roundtrip_low_ids_first_then_lifo():
    m = _mgr(8)
    assert m.allocate(0, 33) == [0, 1, 2]
    assert m.allocate(1, 16) == [3]
    assert m.num_free_blocks == 4
    m.free(0)
    assert m.num_free_blocks == 7
    m.free(1)
    assert m.num_free_blocks == 8
    assert m.allocate(2, 1) == [3]  # freed blocks are reused last-in first-out
    m.check_invariants()


def test_append_crosses_block_boundaries_and_slots_follow_the_table():
    m = _mgr(8)
    m.allocate(0, 15)
    plan = m.schedule([0])
    assert plan.q_lens == [15] and plan.ctx_before == [0]
    slots = m.append_slots(0, 3)
    t = m.block_table(0)
    assert len(t) == 2
    assert slots == [t[0] * BS + 15, t[1] * BS + 0, t[1] * BS + 1]
    plan = m.schedule([0])
    assert plan.ctx_before == [15] and plan.q_lens == [3]
    assert [plan.slot(0, p, BS) for p in range(15, 18)] == slots


def test_out_of_blocks_rolls_back_cleanly():
    m = _mgr(4, cache=True)
    toks = list(range(48))
    m.allocate(0, 48, toks)
    m.schedule([0])
    m.free(0)  # its three full, cached blocks go to the LRU list
    before = (m.num_free_blocks, dict(m._cached))
    with pytest.raises(NoFreeBlocksError):
        m.allocate(1, 100, list(range(1000, 1100)))
    assert not m.has_seq(1)
    assert (m.num_free_blocks, dict(m._cached)) == before
    m.check_invariants()


def test_prefix_hits_only_after_the_writing_step_is_scheduled():
    m = _mgr(300, cache=True)
    p = list(range(1024))
    m.allocate(0, 1024, p)
    m.allocate(1, 1030, p + [7] * 6)  # same step as seq 0: nothing is computed yet
    assert m.num_computed(1) == 0 and m.hits == 0
    plan = m.schedule([0, 1])
    assert plan.q_lens == [1024, 1030]
    m.allocate(2, 1030, p + [9] * 6)  # after the step: 64 blocks come from the cache
    assert m.num_computed(2) == 1024 and m.hits == 64
    assert m.block_table(2)[:64] == m.block_table(0)[:64]
    plan = m.schedule([2])
    assert plan.ctx_before == [1024] and plan.q_lens == [6]


def test_a_full_prompt_hit_recomputes_its_last_block():
    m = _mgr(300, cache=True)
    p = list(range(256))
    m.allocate(0, 256, p)
    m.schedule([0])
    m.allocate(1, 256, p)
    assert m.num_computed(1) == 240  # 15 shared blocks, the 16th is recomputed
    t0, t1 = m.block_table(0), m.block_table(1)
    assert t1[:15] == t0[:15] and t1[15] != t0[15]
    plan = m.schedule([1])
    assert plan.q_lens == [16]


def test_hash_chain_depends_on_everything_before_the_block():
    m = _mgr(300, cache=True)
    a = list(range(64))
    b = [5] + a[1:]  # differs only in the first block
    m.allocate(0, 64, a)
    m.schedule([0])
    m.allocate(1, 80, b + list(range(16)))
    assert m.num_computed(1) == 0, "block 1..3 have equal tokens but a different history"
    m.allocate(2, 80, a + list(range(16)))
    assert m.num_computed(2) == 64


def test_partial_blocks_are_never_shared():
    m = _mgr(300, cache=True)
    p = list(range(40))
    m.allocate(0, 40, p)
    m.schedule([0])
    m.allocate(1, 41, p + [1])
    assert m.num_computed(1) == 32  # two full blocks; block 2 held 8 tokens only
    assert m.block_table(1)[2] != m.block_table(0)[2]


def test_decode_tokens_fill_and_publish_blocks():
    m = _mgr(300, cache=True)
    p = list(range(20))
    m.allocate(0, 20, p)
    m.schedule([0])
    gen = list(range(500, 512))
    m.append_slots(0, 12, gen)  # reaches 32 tokens: block 1 is full
    m.allocate(1, 40, p + gen + [0] * 8)
    assert m.num_computed(1) == 16, "block 1 is not findable before its step is scheduled"
    m.schedule([0])
    m.allocate(2, 40, p + gen + [0] * 8)
    assert m.num_computed(2) == 32


def test_fork_shares_then_copy_on_write_at_the_partial_block():
    m = _mgr(32)
    m.allocate(0, 40)
    m.schedule([0])
    m.fork(0, 1)
    t0 = m.block_table(0)
    assert m.block_table(1) == t0
    assert all(m.refcount[b] == 2 for b in t0)
    s = m.append_slots(1, 1)
    t1 = m.block_table(1)
    assert t1[:2] == t0[:2] and t1[2] != t0[2]
    assert s == [t1[2] * BS + 8]
    plan = m.schedule([1])
    assert plan.copies == [(t0[2], t1[2])]
    assert plan.ctx_before == [40] and plan.q_lens == [1]
    assert m.refcount[t0[2]] == 1 and m.refcount[t1[2]] == 1
    # the parent writes into its own block 2 without a copy
    m.append_slots(0, 1)
    assert m.block_table(0) == t0 and m.schedule([0]).copies == []


def test_a_copy_into_a_released_block_is_dropped():
    m = _mgr(32)
    m.allocate(0, 40)
    m.schedule([0])
    m.fork(0, 1)
    m.append_slots(1, 1)  # queues a copy into the child's new block 2
    assert m.pending_copies
    m.free(1)
    assert m.schedule([0]).copies == []


def test_fork_then_truncate_reuses_a_shared_prefix():
    m = _mgr(300)
    m.allocate(0, 2048)
    m.schedule([0])
    m.fork(0, 1)
    m.truncate_to(1, 1000)  # 62.5 blocks: block 62 is shared and partial
    assert len(m.block_table(1)) == 63
    m.append_slots(1, 24)
    plan = m.schedule([1])
    t0 = m.block_table(0)
    assert plan.copies == [(t0[62], m.block_table(1)[62])]
    assert plan.ctx_before == [1000] and plan.q_lens == [24]
    assert m.block_table(1)[:62] == t0[:62]


def test_fork_before_scheduling_is_refused():
    m = _mgr()
    m.allocate(0, 10)
    with pytest.raises(ValueError):
        m.fork(0, 1)


def test_lru_evicts_oldest_cached_block_after_the_free_list_is_empty():
    m = _mgr(6, cache=True)
    for sid in range(3):  # three single-block prompts + a second block each (17 tokens)
        m.allocate(sid, 17, [sid * 100 + i for i in range(17)])
    m.schedule([0, 1, 2])
    for sid in (1, 0, 2):  # cached first blocks become evictable in this order
        m.free(sid)
    assert len(m._evictable) == 3 and len(m._free) == 3
    m.allocate(10, 48)  # takes the three free blocks first
    assert len(m._evictable) == 3
    m.allocate(11, 16)  # needs one more: evicts seq 1's block (oldest release)
    assert len(m._evictable) == 2
    m.free(10)  # three plain free blocks again: no more evictions needed below
    m.allocate(20, 17, [1 * 100 + i for i in range(17)])
    assert m.num_computed(20) == 0, "seq 1's prefix was evicted"
    m.free(20)
    m.allocate(21, 17, [0 * 100 + i for i in range(17)])
    assert m.num_computed(21) == 16, "seq 0's prefix is still cached"


def test_acquiring_an_evictable_block_takes_it_off_the_lru():
    m = _mgr(8, cache=True)
    p = list(range(33))
    m.allocate(0, 33, p)
    m.schedule([0])
    m.free(0)
    n_evictable = len(m._evictable)
    m.allocate(1, 33, p)
    assert len(m._evictable) == n_evictable - 2
    m.check_invariants()


def test_schedule_rejects_duplicates_and_plans_padding_layout():
    m = _mgr(64)
    m.allocate(0, 5)
    m.allocate(1, 37)
    with pytest.raises(ValueError):
        m.schedule([0, 0])
    plan = m.schedule([0, 1])
    assert plan.query_len == 37 and plan.seq_lens == [5, 37]
    m.append_slots(0, 1)
    plan = m.schedule([0, 1])
    assert plan.q_lens == [1, 0] and plan.query_len == 1


def test_invariant_checker_catches_a_planted_refcount_error():
    m = _mgr(16)
    m.allocate(0, 40)
    m.check_invariants()
    m.refcount[m.block_table(0)[1]] += 1  # planted mistake
    with pytest.raises(AssertionError):
        m.check_invariants()


def test_swap_out_and_in_move_blocks_through_the_next_plan():
    m = BlockManager(16, BS, debug_invariants=True, num_host_blocks=8)
    m.allocate(0, 40)
    m.allocate(1, 20)
    m.schedule([0, 1])
    t0 = m.block_table(0)
    out = m.swap_out(0)
    assert [g for g, _ in out] == t0 and m.is_swapped(0)
    assert m.num_free_host_blocks == 5 and m.num_free_blocks == 16 - 2
    with pytest.raises(ValueError):
        m.schedule([0])
    with pytest.raises(ValueError):
        m.append_slots(0, 1)
    m.append_slots(1, 1)
    plan = m.schedule([1])
    assert plan.swap_out == out and plan.swap_in == []
    back = m.swap_in(0)
    assert [h for h, _ in back] == [h for _, h in out]
    assert not m.is_swapped(0) and m.block_table(0) == [g for _, g in back]
    plan = m.schedule([0])
    assert plan.swap_in == back and plan.q_lens == [0]
    m.append_slots(0, 1)
    assert m.schedule([0]).ctx_before == [40]


def test_swap_needs_scheduled_tokens_and_room():
    m = BlockManager(16, BS, debug_invariants=True, num_host_blocks=2)
    m.allocate(0, 40)
    with pytest.raises(ValueError):
        m.swap_out(0)  # its prompt is not scheduled yet
    m.schedule([0])
    with pytest.raises(NoFreeBlocksError):
        m.swap_out(0)  # three blocks, two host blocks
    assert not m.is_swapped(0) and m.num_free_host_blocks == 2
    m.check_invariants()


def test_swap_in_fails_cleanly_when_hbm_is_full():
    m = BlockManager(4, BS, debug_invariants=True, num_host_blocks=4)
    m.allocate(0, 48)
    m.schedule([0])
    m.swap_out(0)
    m.allocate(1, 64)  # takes every HBM block
    with pytest.raises(NoFreeBlocksError):
        m.swap_in(0)
    assert m.is_swapped(0)
    m.free(1)
    assert len(m.swap_in(0)) == 3


def test_host_blocks_released_by_swap_in_wait_for_the_next_plan():
    m = BlockManager(16, BS, debug_invariants=True, num_host_blocks=2)
    m.allocate(0, 32)
    m.allocate(1, 32)
    m.schedule([0, 1])
    m.swap_out(0)
    m.schedule([1])
    m.swap_in(0)  # releases host blocks that this plan's swap-in still reads
    with pytest.raises(NoFreeBlocksError):
        m.swap_out(1)  # so they cannot be written by a swap-out in the same plan
    plan = m.schedule([0, 1])
    assert len(plan.swap_in) == 2
    assert len(m.swap_out(1)) == 2  # after the plan is built they are free again


def test_swap_in_reuses_blocks_still_cached_in_hbm():
    m = BlockManager(16, BS, enable_prefix_caching=True, debug_invariants=True,
                     num_host_blocks=8)
    toks = list(range(40))
    m.allocate(0, 40, toks)
    m.schedule([0])
    t0 = m.block_table(0)
    m.swap_out(0)
    m.schedule([])
    back = m.swap_in(0)
    # the two full blocks are still cached (evictable) in HBM: only the partial one is copied
    assert len(back) == 1 and m.block_table(0)[:2] == t0[:2]


def test_freeing_a_swapped_sequence_returns_its_host_blocks():
    m = BlockManager(16, BS, debug_invariants=True, num_host_blocks=4)
    m.allocate(0, 40)
    m.schedule([0])
    m.swap_out(0)
    m.free(0)
    plan = m.schedule([])
    assert plan.swap_out == [], "a swap-out of a freed sequence is dropped"
    assert m.num_free_host_blocks == 4


def test_preempt_by_recompute_returns_tokens_and_the_cache_shortens_recompute():
    m = BlockManager(32, BS, enable_prefix_caching=True, debug_invariants=True)
    p = list(range(50))
    m.allocate(0, 50, p)
    m.schedule([0])
    m.append_slots(0, 3, [7, 8, 9])
    m.schedule([0])
    toks = m.preempt(0)
    assert toks == p + [7, 8, 9] and not m.has_seq(0)
    m.allocate(0, len(toks), toks)
    assert m.num_computed(0) == 48


@pytest.mark.parametrize("seed", range(6))
def test_random_operation_sequences_keep_the_invariants(seed):
    """Allocate / append / fork / truncate / free at random under a tight pool."""
    rng = random.Random(seed)
    m = BlockManager(96, BS, enable_prefix_caching=seed % 2 == 0, debug_invariants=True,
                     num_host_blocks=64)
    vocab = 4  # a tiny vocabulary makes shared prefixes common
    live: list[int] = []
    next_id = 0
    for _ in range(400):
        op = rng.random()
        try:
            if op < 0.3 or not live:
                n = rng.randint(1, 120)
                toks = [rng.randrange(vocab) for _ in range(n)]
                # prompts repeat a few canned prefixes
                if rng.random() < 0.5:
                    toks[: min(n, 48)] = [1] * min(n, 48)
                m.allocate(next_id, n, toks)
                live.append(next_id)
                next_id += 1
            elif op < 0.55:
                sid = rng.choice(live)
                m.schedule([sid])
                m.append_slots(sid, rng.randint(1, 20), [rng.randrange(vocab) for _ in range(20)])
            elif op < 0.7:
                sid = rng.choice(live)
                m.schedule([sid])
                m.fork(sid, next_id)
                live.append(next_id)
                next_id += 1
            elif op < 0.8:
                sid = rng.choice(live)
                m.truncate_to(sid, rng.randint(0, m.seq_len(sid)))
            elif op < 0.87:
                resident = [x for x in live if not m.is_swapped(x)]
                plan = m.schedule(rng.sample(resident, k=min(len(resident), 3)))
                for (src, dst) in plan.copies:
                    assert src != dst and m.refcount[dst] >= 1
                hosts_in = {h for h, _ in plan.swap_in}
                assert not hosts_in & {h for _, h in plan.swap_out}
            elif op < 0.93:
                sid = rng.choice(live)
                if m.is_swapped(sid):
                    m.swap_in(sid)
                else:
                    m.schedule([sid])
                    m.swap_out(sid)
            else:
                m.free(live.pop(rng.randrange(len(live))))
        except NoFreeBlocksError:
            if live:
                m.free(live.pop(0))
        except ValueError as e:
            assert "swapped out" in str(e), e
        m.check_invariants()
        for sid in live:
            t = m.block_table(sid)
            assert len(set(t)) == len(t), "a table never repeats a block"
    for sid in live:
        m.free(sid)
    m.schedule([])
    m.check_invariants()
    assert m.num_free_blocks == 96 and m.num_free_host_blocks == 64
