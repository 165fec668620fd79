"""Host-side behaviour of PagedCudaBackend (no GPU needed).

The per-step metadata is built with torch ops on the backend's device; on the
CPU device that logic runs here, while ``forward`` refuses to run (there is no
CPU path). Error types follow the reference's contiguous backend
(pagedserve/attention/contiguous.py:115-121, :180-181).
"""

from __future__ import annotations

import inspect
import os
from pathlib import Path

import pytest
import torch

from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.config import ModelConfig
from paged_serve_b200.interface import AttentionBackend, KVMemoryStats, StepInput

MODEL = ModelConfig("tiny", num_layers=2, num_q_heads=4, num_kv_heads=2, head_dim=64)
# A checkout of the reference project, for the seam-compatibility tests below;
# they are skipped when PAGEDSERVE_REFERENCE is unset.
_REF_ENV = os.environ.get("PAGEDSERVE_REFERENCE", "")
REFERENCE = Path(_REF_ENV) if _REF_ENV else None
NO_REFERENCE = REFERENCE is None or not REFERENCE.exists()


@pytest.fixture
def backend():
    return PagedCudaBackend(MODEL, device="cpu", dtype=torch.bfloat16)


def step(b=2, tq=4, ctx=0, mask=None, seq_lens=None, **kw):
    if mask is None:
        mask = torch.ones((b, ctx + tq), dtype=torch.bool)
    if seq_lens is None:
        seq_lens = mask.sum(1).to(torch.int32)
    return StepInput(query_len=tq, context_len=ctx, seq_lens=seq_lens, padding_mask=mask,
                     is_prefill=tq > 1, **kw)


def test_is_an_attention_backend(backend):
    assert isinstance(backend, AttentionBackend)
    assert backend.name == "paged_cuda"


def test_begin_step_before_allocate_is_runtime_error(backend):
    with pytest.raises(RuntimeError, match="allocate"):
        backend.begin_step(step())


def test_rejects_sequence_longer_than_cache(backend):
    backend.allocate(2, 8)
    with pytest.raises(ValueError, match="exceeds"):
        backend.begin_step(step(tq=16))


def test_rejects_fp32_storage():
    be = PagedCudaBackend(MODEL, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="bf16 or fp16"):
        be.allocate(2, 8)


def test_forward_has_no_cpu_path(backend):
    backend.allocate(2, 16)
    md = backend.begin_step(step())
    q = torch.zeros((2, 4, 4, 64), dtype=torch.bfloat16)
    kv = torch.zeros((2, 4, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        backend.forward(0, q, kv, kv, md)


def test_decode_step_and_new_ops_have_no_cpu_path(backend):
    """The fused decode step, the launch order and the wait self-test refuse CPU
    tensors instead of falling back to a CPU implementation."""
    from paged_serve_b200 import ops

    backend.allocate(2, 16)
    md = backend.begin_step(step(tq=1, ctx=3))
    q = torch.zeros((2, 1, 4, 64), dtype=torch.bfloat16)
    kv = torch.zeros((2, 1, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        backend.forward(0, q, kv, kv, md)
    ctx = torch.tensor([3, 4], dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        ops.decode_order(ctx)
    with pytest.raises(ValueError, match="CUDA"):
        ops.selftest_wait_timeout(torch.zeros(1, dtype=torch.int32))
    pool = torch.zeros((4, 2, 16, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.paged_decode_append(q[:, 0], kv[:, 0], kv[:, 0], torch.zeros(2, dtype=torch.int64),
                                pool, pool, torch.zeros((2, 1), dtype=torch.int32), ctx, 0.1)


def test_left_padded_prefill_metadata(backend):
    backend.allocate(3, 64)
    mask = torch.ones((3, 5), dtype=torch.bool)
    mask[0, :2] = False  # 3 real tokens
    mask[2, :4] = False  # 1 real token
    md = backend.begin_step(step(b=3, tq=5, mask=mask))
    assert md.q_lens.tolist() == [3, 5, 1]
    assert md.ctx_before.tolist() == [0, 0, 0]
    assert md.ctx_lens.tolist() == [3, 5, 1]
    assert md.q_starts.tolist() == [2, 5, 14]
    slots = md.slot_mapping.view(3, 5)
    m = backend.max_blocks_per_seq * 16  # slot i owns blocks [i*M, (i+1)*M)
    assert slots[0].tolist() == [-1, -1, 0, 1, 2]
    assert slots[1].tolist() == [m, m + 1, m + 2, m + 3, m + 4]
    assert slots[2].tolist() == [-1, -1, -1, -1, 2 * m]
    assert md.positions.view(3, 5)[0].tolist() == [-1, -1, 0, 1, 2]


def test_decode_metadata_follows_the_mask(backend):
    backend.allocate(2, 64)
    mask = torch.ones((2, 21), dtype=torch.bool)
    mask[0, :4] = False  # 16 real cached + the new one
    md = backend.begin_step(step(b=2, tq=1, ctx=20, mask=mask))
    assert md.ctx_lens.tolist() == [17, 21]
    assert md.ctx_before.tolist() == [16, 20]
    m = backend.max_blocks_per_seq * 16
    assert md.slot_mapping.tolist() == [16, m + 20]
    assert md.positions.tolist() == [16, 20]


def test_engine_managed_tables_are_used_as_given(backend):
    backend.allocate(2, 64)
    tables = torch.tensor([[7, 3, 0, 0], [1, 2, 5, 6]], dtype=torch.int32)
    slots = torch.tensor([7 * 16 + 5, 6 * 16 + 1], dtype=torch.int64)
    mask = torch.ones((2, 50), dtype=torch.bool)
    mask[0, :44] = False
    md = backend.begin_step(step(b=2, tq=1, ctx=49, mask=mask, block_tables=tables,
                                 slot_mapping=slots))
    assert torch.equal(md.block_tables, tables)
    assert torch.equal(md.slot_mapping, slots)
    assert md.ctx_lens.tolist() == [6, 50]


def test_tables_without_slots_is_value_error(backend):
    backend.allocate(2, 64)
    with pytest.raises(ValueError, match="slot_mapping"):
        backend.begin_step(step(block_tables=torch.zeros((2, 4), dtype=torch.int32)))


def test_debug_invariants_catch_bad_tables():
    be = PagedCudaBackend(MODEL, device="cpu", dtype=torch.bfloat16, num_blocks=16,
                          debug_invariants=True)
    be.allocate(2, 64)
    tables = torch.tensor([[0, 99, 0, 0], [1, 2, 0, 0]], dtype=torch.int32)
    slots = torch.tensor([0, 16], dtype=torch.int64)
    mask = torch.ones((2, 20), dtype=torch.bool)
    with pytest.raises(ValueError, match="block id"):
        be.begin_step(step(b=2, tq=1, ctx=19, mask=mask, block_tables=tables, slot_mapping=slots))
    tables[0, 1] = 3
    with pytest.raises(ValueError, match="one slot twice"):
        be.begin_step(step(b=2, tq=1, ctx=19, mask=mask, block_tables=tables,
                           slot_mapping=torch.tensor([5, 5])))


def test_memory_stats(backend):
    assert backend.memory_stats() == KVMemoryStats(0, 0)
    assert backend.memory_stats().utilization is None
    backend.allocate(2, 64)
    backend.begin_step(step(b=2, tq=10, seq_lens=torch.tensor([10, 10], dtype=torch.int32)))
    stats = backend.memory_stats()
    per_token = 2 * MODEL.num_layers * MODEL.num_kv_heads * MODEL.head_dim * 2
    assert stats.live_bytes == 20 * per_token
    assert stats.allocated_bytes == 2 * 2 * 64 * per_token // 2
    assert stats.utilization == pytest.approx(20 / 128)


def test_memory_stats_with_a_block_manager_use_the_same_reservation():
    """With a block manager, allocated is still the reserved pool (the reference's
    definition, as without one); live counts a prefix block shared through the
    cache once; block_usage gives the blocks sequences hold."""
    be = PagedCudaBackend(MODEL, device="cpu", dtype=torch.bfloat16, num_blocks=64)
    be.allocate(num_seq_slots=4, max_seq_len=256)
    per_token = MODEL.kv_bytes_per_token(torch.bfloat16)
    pool_bytes = 64 * 16 * per_token
    assert be.memory_stats().allocated_bytes == pool_bytes
    mgr = be.make_block_manager(enable_prefix_caching=True)
    prompt = list(range(40))
    mgr.allocate(0, 40, prompt)  # blocks 0, 1 full; block 2 holds 8 tokens
    mgr.schedule([0])
    mgr.allocate(1, 45, prompt[:32] + list(range(100, 113)))  # shares blocks 0 and 1
    st = be.memory_stats()
    assert st.allocated_bytes == pool_bytes
    assert st.live_bytes == (32 + 8 + 13) * per_token
    assert st.utilization == pytest.approx((32 + 8 + 13) / (64 * 16))
    usage = be.block_usage()
    assert usage["held_blocks"] == 4  # seq 0's 3 blocks + seq 1's private third
    assert usage["held_bytes"] == 4 * 16 * per_token
    mgr.free(0)
    mgr.free(1)
    assert be.memory_stats() == KVMemoryStats(pool_bytes, 0)
    assert be.block_usage()["held_blocks"] == 0


def test_standalone_config_kv_bytes_per_token():
    assert MODEL.kv_bytes_per_token(torch.bfloat16) == 2 * 2 * 2 * 64 * 2
    assert MODEL.kv_bytes_per_token(torch.float32) == 2 * 2 * 2 * 64 * 4


def test_free_is_idempotent(backend):
    backend.allocate(2, 16)
    backend.free()
    backend.free()
    assert backend.k_cache is None


@pytest.mark.skipif(NO_REFERENCE, reason="PAGEDSERVE_REFERENCE does not name a reference checkout")
def test_interface_matches_the_reference_seam():
    """Same abstract methods and signatures as pagedserve.attention.backend."""
    import sys

    sys.path.insert(0, str(REFERENCE))
    try:
        import pagedserve.attention.backend as ref
    finally:
        sys.path.remove(str(REFERENCE))
    for name in ("allocate", "free", "begin_step", "forward", "memory_stats"):
        ours = inspect.signature(getattr(AttentionBackend, name))
        theirs = inspect.signature(getattr(ref.AttentionBackend, name))
        assert list(ours.parameters) == list(theirs.parameters), name
        assert list(inspect.signature(getattr(PagedCudaBackend, name)).parameters) == list(
            theirs.parameters), name
    ref_fields = [f for f in ref.StepInput.__dataclass_fields__]
    assert list(StepInput.__dataclass_fields__) == ref_fields
    assert list(KVMemoryStats.__dataclass_fields__) == list(ref.KVMemoryStats.__dataclass_fields__)


@pytest.mark.skipif(NO_REFERENCE, reason="PAGEDSERVE_REFERENCE does not name a reference checkout")
def test_accepts_the_references_own_step_objects(backend):
    import sys

    sys.path.insert(0, str(REFERENCE))
    try:
        import pagedserve.attention.backend as ref
        import pagedserve.config as refcfg
    finally:
        sys.path.remove(str(REFERENCE))
    model = refcfg.ModelConfig(
        name="ref", num_layers=2, hidden_size=256, num_q_heads=4, num_kv_heads=2, head_dim=64,
        intermediate_size=512, vocab_size=10, rms_norm_eps=1e-6, rope_theta=10000.0,
        max_position_embeddings=128, tie_word_embeddings=False, attention_bias=False)
    be = PagedCudaBackend(model, device="cpu", dtype=torch.bfloat16,
                          cache=refcfg.CacheConfig(max_seq_len=64, block_size=16))
    be.allocate(2, 64)
    s = ref.StepInput(query_len=3, context_len=0, seq_lens=torch.tensor([3, 2]),
                      padding_mask=torch.tensor([[1, 1, 1], [0, 1, 1]], dtype=torch.bool),
                      is_prefill=True)
    md = be.begin_step(s)
    assert md.q_lens.tolist() == [3, 2]
    assert be.memory_stats().live_bytes == 5 * model.kv_bytes_per_token(torch.bfloat16)


@pytest.mark.parametrize("pairs,ok", [
    ([(0, 3), (0, 1), (2, 4)], True),
    ([(5, 5)], True),
    ([(0, 3), (3, 1)], False),
    ([(3, 1), (0, 3)], False),
    ([(0, 2), (1, 2)], False),
])
def test_copy_pair_lists_are_checked_like_the_oracle(pairs, ok):
    """ops.check_block_pairs accepts exactly the lists the oracle gives a meaning to."""
    from oracle import oracle_copy_blocks
    from paged_serve_b200.ops import check_block_pairs

    k = torch.zeros(6, 1, 16, 8)
    t = torch.tensor(pairs, dtype=torch.int64)
    if ok:
        check_block_pairs(pairs)
        check_block_pairs(t)
        oracle_copy_blocks(k, k.clone(), t)
    else:
        with pytest.raises(ValueError):
            check_block_pairs(pairs)
        with pytest.raises(ValueError):
            check_block_pairs(t)
        with pytest.raises(ValueError):
            oracle_copy_blocks(k, k.clone(), t)


@pytest.mark.skipif(NO_REFERENCE, reason="PAGEDSERVE_REFERENCE does not name a reference checkout")
def test_is_an_instance_of_the_references_own_seam(backend):
    import sys

    from paged_serve_b200.backend import register_with_reference_seam

    sys.path.insert(0, str(REFERENCE))
    try:
        import pagedserve.attention.backend as ref

        assert register_with_reference_seam()
    finally:
        sys.path.remove(str(REFERENCE))
    assert isinstance(backend, ref.AttentionBackend)
    assert issubclass(PagedCudaBackend, ref.AttentionBackend)


@pytest.mark.parametrize("items,max_keys,pieces", [
    (64, 32768, 9),    # a 512-token chunk of a 32k prompt: 576 units, 97% of 4 waves
    (256, 32768, 4),   # a 2048-token chunk: 1024 units, 99% of 7 waves
    (1, 32768, 16),    # one item: capped at 16 pieces
    (8, 2048, 4),      # capped by 512-key pieces
    (8, 300, 1),       # too short to cut
    (300, 32768, 1),   # two waves already
    (4096, 1536, 1),   # the prefix workload: 27 waves
])
def test_prefill_split_policy(items, max_keys, pieces):
    """Pieces per item from ops.prefill_split_keys on a 148-SM part: the fewest
    that fill whole waves to 90% (else the best fill), pieces of >= 512 keys, at
    most 16, none once the items fill two waves."""
    from paged_serve_b200.ops import prefill_split_keys

    keys = prefill_split_keys(items, max_keys, 148)
    assert keys % 128 == 0
    got = 1 if keys == 0 else -(-max_keys // keys)
    assert got == pieces
    if keys:
        assert keys >= 512
