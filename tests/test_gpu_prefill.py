"""GPU parity: tcgen05 paged prefill against the reference's contiguous prefill.

Covers the reference golden (prefix + causal suffix, GQA 4), random geometries
with every GQA group the kernel tiles (1, 2, 3, 4, 8), lengths that straddle
block and tile boundaries, left-padded and packed query layouts, fp16, and
the full prefix-cached workload (64 sequences over a shared 1024-token
prefix, 8 forking at 1000 with copy-on-write) on a sample of sequences.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_prefill
from paged_serve_b200 import _lib, ops
from paged_serve_b200.workloads import prefix_workload
from tests.conftest import load_golden, pool_from_sequences
from tests.gpu_util import assert_attention_close, random_pool, random_tables

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _prefill(q, kp, vp, tables, q_starts, q_lens, ctx, out=None, err=None):
    d = q.shape[-1]
    return ops.paged_prefill(q, kp, vp, tables, q_starts, q_lens, ctx, int(q_lens.max()),
                             d**-0.5, out=out, device_error=err)


def test_matches_reference_golden():
    g = load_golden("prefill_bf16_gqa4")
    lens = (g["prefix_lens"] + g["q_lens"]).tolist()
    kp = pool_from_sequences(g["keys"], lens, g["block_tables"], g["num_blocks"], 16).to(DEV)
    vp = pool_from_sequences(g["values"], lens, g["block_tables"], g["num_blocks"], 16).to(DEV)
    starts = (torch.cumsum(g["q_lens"], 0) - g["q_lens"]).to(torch.int32)
    out = _prefill(g["query"].to(DEV), kp, vp, g["block_tables"].to(DEV), starts.to(DEV),
                   g["q_lens"].to(DEV), g["prefix_lens"].to(DEV))
    assert_attention_close(out, g["expected"], "prefill golden")


CASES = [
    # (Hq, Hkv, head dim, prefix lens, new lens)
    (32, 8, 128, [0, 1, 15, 16, 17, 100], [1, 33, 64, 65, 127, 129]),  # GQA 4
    (64, 8, 128, [0, 200, 31], [300, 17, 8]),  # GQA 8 (16 tokens per tile)
    (8, 8, 128, [5, 0], [130, 257]),  # MHA (128 tokens per tile)
    (16, 8, 128, [64, 3], [200, 77]),  # GQA 2
    (12, 4, 128, [10, 90], [50, 91]),  # GQA 3 (42 tokens, 126 rows per tile)
    (14, 2, 64, [0, 33, 500], [129, 64, 300]),  # Qwen2.5-0.5B (GQA 7, 18 tokens, 126 rows)
    (32, 8, 64, [16, 0, 1000], [200, 1, 450]),  # GQA 4 at head dim 64
    (32, 2, 128, [0, 77, 300], [100, 9, 64]),  # GQA 16 (8 tokens per tile)
    (24, 2, 128, [40, 0], [150, 33]),  # GQA 12 (10 tokens, 120 rows per tile)
]


@pytest.mark.parametrize("hq,hkv,d,prefix,new", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_random_vs_oracle(hq, hkv, d, prefix, new, dtype):
    bs = 16
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 9
    kp, vp = random_pool(nb, hkv, bs, d, dtype, DEV, seed=hq + hkv)
    tables = random_tables(lens, bs, nb, seed=3, width=max(40, max(lens) // bs + 1))
    gen = torch.Generator(device=DEV).manual_seed(4)
    rows = sum(new)
    q = (torch.randn((rows, hq, d), generator=gen, device=DEV) * 0.5).to(dtype)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = _prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV),
                   err=err)
    assert int(err.item()) == 0
    ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx)
    for i in range(len(new)):
        s = int(starts[i])
        assert_attention_close(out[s : s + new[i]], ref[i], f"hq{hq} seq {i} {dtype}")


@pytest.mark.parametrize("bs", [8, 32])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (14, 2, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_other_block_sizes_vs_oracle(bs, hq, hkv, d, dtype):
    """Block sizes 8 and 32: a 128-key tile is 16 or 4 block boxes."""
    prefix, new = [0, 7, 33, 500], [129, 64, 1, 300]
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 5
    kp, vp = random_pool(nb, hkv, bs, d, dtype, DEV, seed=bs)
    tables = random_tables(lens, bs, nb, seed=7, width=max(lens) // bs + 2)
    gen = torch.Generator(device=DEV).manual_seed(8)
    q = (torch.randn((sum(new), hq, d), generator=gen, device=DEV) * 0.5).to(dtype)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = _prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV),
                   err=err)
    assert int(err.item()) == 0
    ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx)
    for i in range(len(new)):
        s = int(starts[i])
        assert_attention_close(out[s : s + new[i]], ref[i], f"bs{bs} hq{hq} seq {i}")


SPLIT_CASES = [
    # (Hq, Hkv, head dim, block size, prefix lens, new lens, keys per piece)
    (32, 8, 128, 16, [3000, 0, 17], [200, 129, 64], 512),  # a long item in 7 pieces, short ones whole
    (8, 8, 128, 16, [0, 300], [257, 130], 128),  # MHA: tile A rows see no key in tile B's piece
    (14, 2, 64, 16, [2500, 33], [129, 300], 384),  # head dim 64, GQA 7
    (32, 2, 128, 8, [1000, 5], [100, 40], 256),  # GQA 16, 8-token blocks
    (16, 8, 128, 32, [4000], [77], 1024),  # GQA 2, 32-token blocks
]


@pytest.mark.parametrize("hq,hkv,d,bs,prefix,new,split", SPLIT_CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_split_k_vs_oracle_and_whole_items(hq, hkv, d, bs, prefix, new, split, dtype):
    """ps_paged_prefill_split: items cut into key-range pieces and merged agree
    with the oracle and with the unsplit kernel; rows owned by no sequence stay
    untouched."""
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 9
    kp, vp = random_pool(nb, hkv, bs, d, dtype, DEV, seed=hq + bs)
    tables = random_tables(lens, bs, nb, seed=5, width=max(lens) // bs + 3)
    gen = torch.Generator(device=DEV).manual_seed(6)
    tq = max(new) + 3  # left-padded [B, tq] rows
    q = (torch.randn((len(new) * tq, hq, d), generator=gen, device=DEV) * 0.5).to(dtype)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = torch.tensor([b * tq + tq - n for b, n in enumerate(new)], dtype=torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = (q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV), tq, d**-0.5)
    need = ops.prefill_workspace_bytes(len(new), tq, hq, hkv, d, bs, tables.shape[1], split)
    assert need > 0
    ws = torch.full((need,), 0xFF, dtype=torch.uint8, device=DEV)  # NaN-filled partials
    got = ops.paged_prefill(*args, out=torch.full_like(q, 7.0), device_error=err,
                            split_keys=split, workspace=ws)
    whole = ops.paged_prefill(*args, device_error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx)
    for i in range(len(new)):
        s = int(starts[i])
        assert_attention_close(got[s : s + new[i]], ref[i], f"split hq{hq} bs{bs} seq {i}")
        assert_attention_close(got[s : s + new[i]], whole[s : s + new[i]].float(),
                               f"split vs whole seq {i}")
        assert bool((got[i * tq : s] == 7.0).all())


def test_split_k_workspace_reused_by_a_larger_call_and_max_keys_bound():
    """A second, larger split call over the first call's partials; ``max_keys``
    narrows the pieces (and the workspace) below what the table width allows."""
    hq, hkv, d, bs = 32, 8, 128, 16
    width = 512  # 8192 keys
    calls = ((1, [1500], [90]), (2, [5000, 2200], [300, 64]))
    needs = []
    for _, prefix, new in calls:
        lens = [p + n for p, n in zip(prefix, new, strict=True)]
        narrow = ops.prefill_workspace_bytes(len(new), max(new), hq, hkv, d, bs,
                                             -(-max(lens) // bs), 512)
        wide = ops.prefill_workspace_bytes(len(new), max(new), hq, hkv, d, bs, width, 512)
        assert 0 < narrow < wide
        needs.append(narrow)
    assert needs[1] > needs[0]
    ws = torch.empty(needs[1], dtype=torch.uint8, device=DEV)  # shared by both calls
    for seed, prefix, new in calls:
        lens = [p + n for p, n in zip(prefix, new, strict=True)]
        nb = sum((n + bs - 1) // bs for n in lens) + 4
        kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=seed)
        tables = random_tables(lens, bs, nb, seed=seed, width=width)
        q = (torch.randn((sum(new), hq, d), device=DEV) * 0.5).to(torch.bfloat16)
        q_lens = torch.tensor(new, dtype=torch.int32)
        starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
        ctx = torch.tensor(prefix, dtype=torch.int32)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        got = ops.paged_prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV),
                                ctx.to(DEV), max(new), d**-0.5, device_error=err,
                                split_keys=512, workspace=ws, max_keys=max(lens))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx)
        for i in range(len(new)):
            s = int(starts[i])
            assert_attention_close(got[s : s + new[i]], ref[i], f"call {seed} seq {i}")


def test_left_padded_layout_leaves_pad_rows_untouched():
    """Rows of a padded [B, Tq] layout that belong to no sequence are not written."""
    hq, hkv, d, bs, tq = 32, 8, 128, 16, 40
    new = [40, 23, 1]
    prefix = [7, 0, 300]
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = 40
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=8)
    tables = random_tables(lens, bs, nb, seed=9, width=24)
    q = (torch.randn((3 * tq, hq, d), device=DEV) * 0.5).to(torch.bfloat16)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = torch.tensor([b * tq + tq - n for b, n in enumerate(new)], dtype=torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    sentinel = torch.full_like(q, 7.0)
    out = _prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV),
                   out=sentinel)
    ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx)
    for i in range(3):
        s = int(starts[i])
        assert_attention_close(out[s : s + new[i]], ref[i], f"padded seq {i}")
        pad = out[i * tq : s]
        assert bool((pad == 7.0).all())


def test_sequences_without_new_tokens_and_a_long_prompt():
    """Sequences with no new tokens (their rows are untouched) next to a 2300-token
    prompt with no prefix (many query tiles, the causal diagonal in every one)."""
    hq, hkv, d, bs = 32, 8, 128, 16
    new = [0, 2300, 0, 33, 0]
    prefix = [50, 0, 0, 1000, 7]
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 5
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=21)
    tables = random_tables(lens, bs, nb, seed=22, width=max(lens) // bs + 1)
    rows = sum(new)
    q = (torch.randn((rows, hq, d), generator=torch.Generator().manual_seed(23)) * 0.5).to(
        torch.bfloat16).to(DEV)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = _prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV),
                   err=err)
    assert int(err.item()) == 0
    ref = oracle_prefill(q, kp, vp, tables, starts, q_lens, ctx, seqs=[1, 3])
    for i in (1, 3):
        s = int(starts[i])
        assert_attention_close(out[s : s + new[i]], ref[i], f"seq {i}")


def test_block_placement_is_bit_invariant():
    """Relocating every block of the pool (tables rewritten to match) leaves the
    output bit-identical: placement only changes where the TMA reads."""
    hq, hkv, d, bs = 32, 8, 128, 16
    new = [300, 129, 512]
    prefix = [1000, 17, 0]
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 20
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=31)
    tables = random_tables(lens, bs, nb, seed=32, width=max(lens) // bs + 1)
    q = (torch.randn((sum(new), hq, d), generator=torch.Generator().manual_seed(33)) * 0.5).to(
        torch.bfloat16).to(DEV)
    q_lens = torch.tensor(new, dtype=torch.int32, device=DEV)
    starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32, device=DEV)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(34)).to(DEV)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(nb, device=DEV)
    moved = inv[tables.to(DEV).long()].to(torch.int32)
    a = _prefill(q, kp, vp, tables.to(DEV), starts, q_lens, ctx)
    b = _prefill(q, kp[perm], vp[perm], moved, starts, q_lens, ctx)
    assert torch.equal(a, b)


def test_query_and_out_as_views_of_fused_buffers():
    """q is the Q slice of a fused [T, (Hq + 2 Hkv) * D] projection and out a slice of a
    wider buffer: token strides larger than Hq * D, columns outside untouched."""
    hq, hkv, d, bs = 16, 4, 128, 16
    new = [70, 200]
    prefix = [33, 0]
    lens = [p + n for p, n in zip(prefix, new, strict=True)]
    nb = sum((n + bs - 1) // bs for n in lens) + 3
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=41)
    tables = random_tables(lens, bs, nb, seed=42)
    t = sum(new)
    fused = (torch.randn((t, (hq + 2 * hkv) * d), generator=torch.Generator().manual_seed(43))
             * 0.5).to(torch.bfloat16).to(DEV)
    q = fused[:, : hq * d].view(t, hq, d)
    wide = torch.zeros((t, 2 * hq * d), dtype=torch.bfloat16, device=DEV)
    out = wide[:, hq * d :].view(t, hq, d)
    q_lens = torch.tensor(new, dtype=torch.int32)
    starts = (torch.cumsum(q_lens, 0) - q_lens).to(torch.int32)
    ctx = torch.tensor(prefix, dtype=torch.int32)
    _prefill(q, kp, vp, tables.to(DEV), starts.to(DEV), q_lens.to(DEV), ctx.to(DEV), out=out)
    assert torch.count_nonzero(wide[:, : hq * d]) == 0
    ref = oracle_prefill(q.contiguous(), kp, vp, tables, starts, q_lens, ctx)
    for i in range(2):
        s = int(starts[i])
        assert_attention_close(out[s : s + new[i]], ref[i], f"fused seq {i}")


def test_bad_block_id_is_reported():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.tensor([[0, 1, 8 + 3, 2]], dtype=torch.int32, device=DEV)
    q = torch.randn((20, 8, 128), device=DEV).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    one = torch.tensor([0], dtype=torch.int32, device=DEV)
    _prefill(q, kp, vp, tables, one * 0, one * 0 + 20, one * 0 + 40, err=err)
    assert int(err.item()) & _lib.PS_DEVERR_BLOCK_ID


def test_rows_out_of_range_are_reported_not_written():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.arange(8, dtype=torch.int32, device=DEV).view(1, 8)
    q = torch.randn((10, 8, 128), device=DEV).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.zeros_like(q)
    ops.paged_prefill(q, kp, vp, tables, torch.tensor([5], dtype=torch.int32, device=DEV),
                      torch.tensor([8], dtype=torch.int32, device=DEV),
                      torch.tensor([0], dtype=torch.int32, device=DEV), 8, 0.1, out=out,
                      device_error=err)
    assert int(err.item()) & _lib.PS_DEVERR_LENGTH
    assert torch.count_nonzero(out) == 0


def test_split_k_reports_bad_block_ids_and_rows_out_of_range():
    """The split-K kernel and its merge keep the whole-item kernel's guards: a
    block id past the pool in one piece sets PS_DEVERR_BLOCK_ID (the read is
    redirected to a valid block), and rows past the query buffer set
    PS_DEVERR_LENGTH with nothing written by either launch."""
    kp, vp = random_pool(40, 2, 16, 128, torch.bfloat16, DEV, seed=1)
    tables = torch.arange(20, dtype=torch.int32).view(1, 20)
    tables[0, 12] = 40 + 3  # keys 192-207: the second of three 128-key pieces
    q = torch.randn((20, 8, 128), device=DEV).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    one = torch.tensor([1], dtype=torch.int32, device=DEV)
    ops.paged_prefill(q, kp, vp, tables.to(DEV), one * 0, one * 20, one * 300, 20, 0.1,
                      device_error=err, split_keys=128)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.PS_DEVERR_BLOCK_ID

    err.zero_()
    q = torch.randn((10, 8, 128), device=DEV).to(torch.bfloat16)
    out = torch.zeros_like(q)
    tables = torch.arange(24, dtype=torch.int32, device=DEV).view(1, 24)  # up to 3 pieces
    ops.paged_prefill(q, kp, vp, tables, one * 5, one * 8, one * 0, 8, 0.1, out=out,
                      device_error=err, split_keys=128)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.PS_DEVERR_LENGTH
    assert torch.count_nonzero(out) == 0


@pytest.fixture(scope="module")
def prefix_case():
    wl = prefix_workload(seed=0)
    dtype = torch.bfloat16
    gen = torch.Generator(device=DEV).manual_seed(0)
    shape = (wl.num_blocks, wl.num_kv_heads, wl.block_size, wl.head_dim)
    kp = torch.empty(shape, dtype=dtype, device=DEV).normal_(0, 0.5, generator=gen)
    vp = torch.empty(shape, dtype=dtype, device=DEV).normal_(0, 0.5, generator=gen)
    q = torch.empty((wl.total_q, wl.num_q_heads, wl.head_dim), dtype=dtype,
                    device=DEV).normal_(0, 0.5, generator=gen)
    k_new = torch.empty((wl.total_q, wl.num_kv_heads, wl.head_dim), dtype=dtype,
                        device=DEV).normal_(0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    # copy-on-write of the partially shared block, then the suffix append
    ops.copy_blocks(kp, vp, wl.cow_pairs.to(DEV))
    ops.cache_append(kp, vp, k_new, v_new, wl.slot_mapping.to(DEV))
    return wl, q, kp, vp


def test_prefix_workload_sample_vs_oracle(prefix_case):
    wl, q, kp, vp = prefix_case
    out = _prefill(q, kp, vp, wl.block_tables.to(DEV), wl.q_starts.to(DEV), wl.q_lens.to(DEV),
                   wl.prefix_lens.to(DEV))
    sample = [0, 1, 31, 55, 56, 57, 63]  # 56..63 forked at 1000 through a CoW block
    ref = oracle_prefill(q, kp, vp, wl.block_tables, wl.q_starts, wl.q_lens, wl.prefix_lens,
                         seqs=sample)
    for i in sample:
        s = int(wl.q_starts[i])
        assert_attention_close(out[s : s + 512], ref[i], f"prefix seq {i}")


def test_prefix_workload_every_sequence_vs_oracle_on_gpu(prefix_case):
    """All 64 sequences (8 forked through a copy-on-write block) against the
    oracle's steps run on the GPU in fp32."""
    wl, q, kp, vp = prefix_case
    out = _prefill(q, kp, vp, wl.block_tables.to(DEV), wl.q_starts.to(DEV), wl.q_lens.to(DEV),
                   wl.prefix_lens.to(DEV))
    ref = oracle_prefill(q, kp, vp, wl.block_tables, wl.q_starts, wl.q_lens, wl.prefix_lens,
                         device=DEV)
    for i in range(wl.batch):
        s = int(wl.q_starts[i])
        assert_attention_close(out[s : s + 512], ref[i], f"prefix seq {i} (GPU oracle)")


def test_prefix_workload_is_bit_deterministic_and_shared_prefix_consistent(prefix_case):
    """Two runs agree bit-for-bit; sequences with identical inputs give identical rows."""
    wl, q, kp, vp = prefix_case
    args = (wl.block_tables.to(DEV), wl.q_starts.to(DEV), wl.q_lens.to(DEV),
            wl.prefix_lens.to(DEV))
    a = _prefill(q, kp, vp, *args)
    b = _prefill(q, kp, vp, *args)
    assert torch.equal(a, b)
