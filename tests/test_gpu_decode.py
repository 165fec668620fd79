"""GPU parity: paged decode attention against the reference's contiguous path.

Small cases run the oracle on every sequence; the full Llama-3-8B-shaped layer
(256 sequences, ctx up to 4096) checks a sample of sequences against the oracle
and the whole batch through size-independent properties (block placement
invariance, split-K consistency).
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_decode
from paged_serve_b200 import _lib, ops
from paged_serve_b200.workloads import decode_workload, fill_pool
from tests.conftest import load_golden, pool_from_sequences
from tests.gpu_util import (
    assert_attention_close,
    oracle_decode_on_device,
    random_pool,
    random_tables,
)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _decode(q, kp, vp, tables, ctx, split, err=None):
    hq, d = q.shape[1], q.shape[2]
    ws = None
    if split:
        nbytes = ops.decode_workspace_bytes(q.shape[0], hq, d, kp.shape[2], tables.shape[1], split)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
    return ops.paged_decode(q, kp, vp, tables, ctx, 1.0 / d**0.5, split, workspace=ws,
                            device_error=err)


@pytest.mark.parametrize("name", ["decode_bf16_gqa4", "decode_bf16_gqa7"])
@pytest.mark.parametrize("split", [0, 16, 64])
def test_matches_reference_golden(name, split):
    g = load_golden(name)
    lens = g["ctx_lens"].tolist()
    kp = pool_from_sequences(g["keys"], lens, g["block_tables"], g["num_blocks"], 16).to(DEV)
    vp = pool_from_sequences(g["values"], lens, g["block_tables"], g["num_blocks"], 16).to(DEV)
    out = _decode(g["query"].to(DEV), kp, vp, g["block_tables"].to(DEV), g["ctx_lens"].to(DEV),
                  split)
    assert_attention_close(out, g["expected"], name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("split", [0, 16, 64])
def test_cpu_plumbing_case_on_the_gpu(dtype, split):
    """The reference's fp32 plumbing case (Hq 8, Hkv 2, D 64, contexts {17, 64, 100, 255},
    a 128-block pool, shuffled tables) run through the kernel in 16-bit: it must match
    the oracle on the same rounded inputs, and the fixture's fp32 output within the
    extra error the input rounding brings."""
    g = load_golden("tiny_decode")
    lens = g["ctx_lens"].tolist()
    kp = pool_from_sequences(g["keys"], lens, g["block_tables"], g["num_blocks"], 16).to(dtype)
    vp = pool_from_sequences(g["values"], lens, g["block_tables"], g["num_blocks"], 16).to(dtype)
    q = g["query"].to(dtype)
    out = _decode(q.to(DEV), kp.to(DEV), vp.to(DEV), g["block_tables"].to(DEV),
                  g["ctx_lens"].to(DEV), split)
    ref = oracle_decode(q, kp, vp, g["block_tables"], g["ctx_lens"])
    assert_attention_close(out, ref, f"tiny_decode {dtype} split {split}")
    # N(0,1) inputs rounded to 16 bits move the fp32 answer by a few 1e-3 at most
    assert float((out.float().cpu() - g["expected"]).abs().max()) < 3e-2


GEOMS = [
    (32, 8, 128),  # Llama-3-8B (GQA 4)
    (64, 8, 128),  # Llama-3-70B (GQA 8)
    (8, 8, 128),  # MHA
    (14, 2, 64),  # Qwen2.5-0.5B (GQA 7)
    (12, 4, 64),  # GQA 3
    (32, 2, 128),  # GQA 16 (rows 8-15 of the MMA carried)
    (24, 2, 128),  # GQA 12 (Mistral-Large's ratio)
    (18, 2, 64),  # GQA 9
]


@pytest.mark.parametrize("hq,hkv,d", GEOMS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("split", [0, 64, 512])
def test_random_batches_vs_oracle(hq, hkv, d, dtype, split):
    lens = [1, 2, 15, 16, 17, 31, 32, 33, 64, 100, 511, 512, 513, 1000, 1500, 2049]
    bs = 16
    nb = sum((n + bs - 1) // bs for n in lens) + 37
    kp, vp = random_pool(nb, hkv, bs, d, dtype, DEV, seed=hq * 7 + d)
    tables = random_tables(lens, bs, nb, seed=1, width=160)
    gen = torch.Generator(device=DEV).manual_seed(2)
    q = (torch.randn((len(lens), hq, d), generator=gen, device=DEV) * 0.5).to(dtype)
    ctx = torch.tensor(lens, dtype=torch.int32)
    out = _decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), split)
    ref = oracle_decode(q, kp, vp, tables, ctx)
    assert_attention_close(out, ref, f"hq{hq} hkv{hkv} d{d} {dtype} split{split}")


@pytest.mark.parametrize("bs", [8, 32])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (14, 2, 64), (32, 2, 128)])
@pytest.mark.parametrize("split", [0, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_other_block_sizes_vs_oracle(bs, hq, hkv, d, split, dtype):
    """Block sizes 8 and 32 (the reference sweeps CacheConfig.block_size): a 16-key chunk
    is two 8-row blocks or half of a 32-row block."""
    lens = [1, 7, 8, 9, 15, 16, 17, 31, 32, 33, 100, 257, 1000]
    nb = sum((n + bs - 1) // bs for n in lens) + 11
    kp, vp = random_pool(nb, hkv, bs, d, dtype, DEV, seed=bs + d)
    tables = random_tables(lens, bs, nb, seed=5, width=1024 // bs + 2)
    gen = torch.Generator(device=DEV).manual_seed(6)
    q = (torch.randn((len(lens), hq, d), generator=gen, device=DEV) * 0.5).to(dtype)
    ctx = torch.tensor(lens, dtype=torch.int32)
    out = _decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), split)
    ref = oracle_decode(q, kp, vp, tables, ctx)
    assert_attention_close(out, ref, f"bs{bs} hq{hq} d{d} split{split}")


def test_split_workspace_reused_across_calls():
    """Split-K plans its (sequence, partition) units and resets its claim counter in
    the workspace on every call: one workspace serves calls with different length
    sets (empty sequences, 1 to 64 partitions) back to back, each matching the oracle."""
    hq, hkv, d, bs, split = 16, 2, 128, 16, 64
    width = 4096 // bs
    nb = 64 * width + 16  # room for 64 sequences at the longest length
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=11)
    nbytes = ops.decode_workspace_bytes(64, hq, d, bs, width, split)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    gen = torch.Generator().manual_seed(12)
    for call, lens in enumerate([
        [0, 1, 64, 65, 4000, 129, 0, 3],
        [4033, 17, 2000, 64] * 4,
        [int(x) for x in torch.randint(0, 4097, (64,), generator=gen)],
    ]):
        tables = random_tables(lens, bs, nb, seed=13 + call, width=width)
        q = (torch.randn((len(lens), hq, d), generator=gen) * 0.5).to(torch.bfloat16).to(DEV)
        ctx = torch.tensor(lens, dtype=torch.int32)
        out = ops.paged_decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), d**-0.5, split, workspace=ws)
        ref = oracle_decode(q, kp, vp, tables, ctx)
        assert_attention_close(out, ref, f"call {call}")
        for i, n in enumerate(lens):
            if n == 0:
                assert torch.count_nonzero(out[i]) == 0


def test_decode_order_is_a_longest_first_permutation():
    gen = torch.Generator().manual_seed(51)
    for lens in ([0], [5, 5, 5], [int(x) for x in torch.randint(0, 40000, (3000,), generator=gen)]):
        ctx = torch.tensor(lens, dtype=torch.int32)
        order = ops.decode_order(ctx.to(DEV)).cpu()
        assert sorted(order.tolist()) == list(range(len(lens)))
        # non-increasing up to the sort's bucket width (1/1024 of the longest + 1)
        width = (max(lens) + 1) / 1024
        ranked = ctx[order.long()]
        assert bool((ranked[1:] <= ranked[:-1] + width).all())


@pytest.mark.parametrize("split", [0, 64])
def test_launch_order_does_not_change_the_result(split):
    """Longest-first order (and any other permutation) gives bit-identical outputs."""
    hq, hkv, d, bs = 32, 8, 128, 16
    lens = [3000, 1, 700, 0, 4096, 64, 1500, 17, 2222, 900]
    nb = sum((n + bs - 1) // bs for n in lens) + 7
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=52)
    tables = random_tables(lens, bs, nb, seed=53, width=4096 // bs).to(DEV)
    q = (torch.randn((len(lens), hq, d), generator=torch.Generator().manual_seed(54)) * 0.5).to(
        torch.bfloat16).to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    ws = torch.empty(max(ops.decode_workspace_bytes(len(lens), hq, d, bs, 4096 // bs, split), 256),
                     dtype=torch.uint8, device=DEV)
    base = ops.paged_decode(q, kp, vp, tables, ctx, d**-0.5, split, workspace=ws)
    for order in (ops.decode_order(ctx),
                  torch.randperm(len(lens), generator=torch.Generator().manual_seed(55)).to(
                      torch.int32).to(DEV)):
        got = ops.paged_decode(q, kp, vp, tables, ctx, d**-0.5, split, workspace=ws,
                               seq_order=order)
        assert torch.equal(got, base)


def test_bad_launch_order_entry_is_reported():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.arange(8, dtype=torch.int32, device=DEV).view(2, 4)
    q = torch.randn((2, 8, 128), device=DEV).to(torch.bfloat16)
    ctx = torch.tensor([40, 20], dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    order = torch.tensor([1, 7], dtype=torch.int32, device=DEV)  # 7 is not a sequence
    ops.paged_decode(q, kp, vp, tables, ctx, 0.1, 0, device_error=err, seq_order=order)
    assert int(err.item()) & _lib.PS_DEVERR_LENGTH


@pytest.mark.parametrize("split", [0, 64])
@pytest.mark.parametrize("bs,hq,hkv,d", [(16, 32, 8, 128), (8, 32, 2, 128), (32, 14, 2, 64)])
def test_fused_append_equals_append_then_decode(split, bs, hq, hkv, d):
    """ps_paged_decode_append leaves the same pools and returns the same output,
    bit for bit, as ps_cache_append followed by ps_paged_decode (padding rows with
    slot -1 included)."""
    # keys after the step (0 = padding row); 128 and 2048 end exactly on a 64-token
    # partition, 2049 opens a one-token last partition
    lens = [1, 17, 700, 16, 2049, 33, 0, 400, 128, 2048]
    nb = sum((n + bs - 1) // bs for n in lens) + 9
    kp, vp = random_pool(nb, hkv, bs, d, torch.bfloat16, DEV, seed=61)
    width = 4096 // bs
    tables = random_tables(lens, bs, nb, seed=62, width=width)
    slots = torch.tensor([int(tables[i, (n - 1) // bs]) * bs + (n - 1) % bs if n else -1
                          for i, n in enumerate(lens)], dtype=torch.int64)
    gen = torch.Generator().manual_seed(63)
    q = (torch.randn((len(lens), hq, d), generator=gen) * 0.5).to(torch.bfloat16).to(DEV)
    k_new = torch.randn((len(lens), hkv, d), generator=gen).to(torch.bfloat16).to(DEV)
    v_new = torch.randn((len(lens), hkv, d), generator=gen).to(torch.bfloat16).to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    tables, slots = tables.to(DEV), slots.to(DEV)
    ws = torch.empty(max(ops.decode_workspace_bytes(len(lens), hq, d, bs, width, split), 256),
                     dtype=torch.uint8, device=DEV)
    order = ops.decode_order(ctx)
    k1, v1 = kp.clone(), vp.clone()
    ops.cache_append(k1, v1, k_new, v_new, slots)
    ref = ops.paged_decode(q, k1, v1, tables, ctx, d**-0.5, split, workspace=ws, seq_order=order)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = ops.paged_decode_append(q, k_new, v_new, slots, kp, vp, tables, ctx, d**-0.5, split,
                                  workspace=ws, device_error=err, seq_order=order)
    assert int(err.item()) == 0
    assert torch.equal(kp, k1) and torch.equal(vp, v1)
    assert torch.equal(got, ref)


def test_fused_append_bad_slot_is_reported_not_written():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    before_k, before_v = kp.clone(), vp.clone()
    tables = torch.arange(8, dtype=torch.int32, device=DEV).view(2, 4)
    q = torch.randn((2, 8, 128), device=DEV).to(torch.bfloat16)
    k_new = torch.randn((2, 2, 128), device=DEV).to(torch.bfloat16)
    ctx = torch.tensor([40, 20], dtype=torch.int32, device=DEV)
    slots = torch.tensor([-1, 8 * 16 + 5], dtype=torch.int64, device=DEV)  # past the pool
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.paged_decode_append(q, k_new, k_new, slots, kp, vp, tables, ctx, 0.1, 0,
                            device_error=err)
    assert int(err.item()) & _lib.PS_DEVERR_SLOT
    assert torch.equal(kp, before_k) and torch.equal(vp, before_v)


def test_zero_context_outputs_zeros():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.arange(8, dtype=torch.int32).view(2, 4)
    q = torch.randn((2, 8, 128), device=DEV).to(torch.bfloat16)
    ctx = torch.tensor([0, 40], dtype=torch.int32)
    for split in (0, 16):
        out = _decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), split)
        assert torch.count_nonzero(out[0]) == 0
        assert_attention_close(out[1], oracle_decode(q, kp, vp, tables, ctx)[1], "ctx40")


def test_scattered_q_and_out_strides():
    """q and out as row views of a larger [B, 3*Hq*D] buffer."""
    b, hq, hkv, d = 5, 32, 8, 128
    lens = [7, 300, 16, 1024, 65]
    nb = 120
    kp, vp = random_pool(nb, hkv, 16, d, torch.bfloat16, DEV, seed=4)
    tables = random_tables(lens, 16, nb, seed=5)
    buf = torch.randn((b, 3 * hq * d), device=DEV).to(torch.bfloat16)
    q = buf[:, hq * d : 2 * hq * d].view(b, hq, d)
    obuf = torch.zeros((b, 2 * hq * d), dtype=torch.bfloat16, device=DEV)
    out = obuf[:, hq * d :].view(b, hq, d)
    ctx = torch.tensor(lens, dtype=torch.int32)
    ops.paged_decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), d**-0.5, 0, out=out)
    assert torch.count_nonzero(obuf[:, : hq * d]) == 0
    assert_attention_close(out, oracle_decode(q, kp, vp, tables, ctx), "strided")


def test_bad_block_id_reports_error_instead_of_faulting():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.tensor([[0, 1, 8 + 5]], dtype=torch.int32, device=DEV)
    q = torch.randn((1, 8, 128), device=DEV).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _decode(q, kp, vp, tables, torch.tensor([40], dtype=torch.int32, device=DEV), 0, err)
    assert int(err.item()) & _lib.PS_DEVERR_BLOCK_ID


def test_context_longer_than_table_reports_error():
    kp, vp = random_pool(8, 2, 16, 128, torch.bfloat16, DEV, seed=0)
    tables = torch.tensor([[0, 1]], dtype=torch.int32, device=DEV)
    q = torch.randn((1, 8, 128), device=DEV).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = _decode(q, kp, vp, tables, torch.tensor([33], dtype=torch.int32, device=DEV), 0, err)
    assert int(err.item()) & _lib.PS_DEVERR_LENGTH
    assert torch.count_nonzero(out) == 0


@pytest.fixture(scope="module")
def llama8b_layer():
    wl = decode_workload("llama8b", seed=0)
    kp, vp = fill_pool(wl.num_blocks, wl.spec, torch.bfloat16, torch.device(DEV), seed=0)
    gen = torch.Generator(device=DEV).manual_seed(1)
    q = torch.empty((wl.batch, wl.spec.num_q_heads, wl.spec.head_dim), dtype=torch.bfloat16,
                    device=DEV).normal_(0.0, 0.5, generator=gen)
    return wl, q, kp[0], vp[0]


@pytest.mark.parametrize("split", [0, 512, 1024])
def test_llama8b_full_layer_sample_vs_oracle(llama8b_layer, split):
    wl, q, kp, vp = llama8b_layer
    tables = wl.block_tables.to(DEV)
    ctx = wl.ctx_lens.to(DEV)
    out = _decode(q, kp, vp, tables, ctx, split)
    sample = [0, 1, 17, 64, 100, 128, 200, 255] + torch.argsort(wl.ctx_lens)[-4:].tolist()
    ref = oracle_decode(q[sample], kp, vp, wl.block_tables[sample], wl.ctx_lens[sample])
    assert_attention_close(out[sample], ref, f"llama8b split{split}")


@pytest.mark.parametrize("split", [0, 512])
def test_llama8b_full_layer_every_sequence_vs_oracle_on_gpu(llama8b_layer, split):
    """All 256 sequences of the full layer against the oracle's steps run on the GPU in fp32."""
    wl, q, kp, vp = llama8b_layer
    out = _decode(q, kp, vp, wl.block_tables.to(DEV), wl.ctx_lens.to(DEV), split)
    ref = oracle_decode_on_device(q, kp, vp, wl.block_tables, wl.ctx_lens)
    assert_attention_close(out, ref, f"llama8b every sequence, split {split}")


def test_llama8b_split_and_unsplit_agree(llama8b_layer):
    wl, q, kp, vp = llama8b_layer
    tables, ctx = wl.block_tables.to(DEV), wl.ctx_lens.to(DEV)
    a = _decode(q, kp, vp, tables, ctx, 0).float()
    b = _decode(q, kp, vp, tables, ctx, 512).float()
    assert_attention_close(b, a, "split vs unsplit")


def test_llama8b_block_placement_is_bit_invariant(llama8b_layer):
    """Relocating every block (permuting the pool) leaves the output bit-identical."""
    wl, q, kp, vp = llama8b_layer
    perm = torch.randperm(wl.num_blocks, generator=torch.Generator().manual_seed(3)).to(DEV)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(wl.num_blocks, device=DEV)
    tables = wl.block_tables.to(DEV)
    moved = inv[tables.long()].to(torch.int32)
    ctx = wl.ctx_lens.to(DEV)
    for split in (0, 512):
        a = _decode(q, kp, vp, tables, ctx, split)
        b = _decode(q, kp[perm], vp[perm], moved, ctx, split)
        assert torch.equal(a, b)


@pytest.fixture(scope="module")
def llama70b_layer():
    """One layer of the long-context skewed 70B decode: 512 sequences, lengths
    lognormal (median 2048, sigma 1) clipped to [128, 32768], GQA 8."""
    wl = decode_workload("llama70b", seed=0)
    kp, vp = fill_pool(wl.num_blocks, wl.spec, torch.bfloat16, torch.device(DEV), seed=0)
    gen = torch.Generator(device=DEV).manual_seed(1)
    q = torch.empty((wl.batch, wl.spec.num_q_heads, wl.spec.head_dim), dtype=torch.bfloat16,
                    device=DEV).normal_(0.0, 0.5, generator=gen)
    return wl, q, kp[0], vp[0]


def _compact_pool(wl, sample, kp, vp):
    """The sampled sequences' blocks as a small pool with renumbered tables, so the
    oracle (which copies its pool to the host) reads megabytes, not the whole layer.
    Block placement does not change the decode's bits (tested above)."""
    bs = wl.spec.block_size
    rows = [wl.block_tables[i, : (int(wl.ctx_lens[i]) + bs - 1) // bs].long() for i in sample]
    uniq, inv = torch.unique(torch.cat(rows), return_inverse=True)
    tables = torch.zeros((len(sample), max(r.numel() for r in rows)), dtype=torch.int32)
    at = 0
    for j, r in enumerate(rows):
        tables[j, : r.numel()] = inv[at : at + r.numel()].to(torch.int32)
        at += r.numel()
    idx = uniq.to(DEV)
    return kp[idx], vp[idx], tables


def test_llama70b_full_layer_sample_vs_oracle(llama70b_layer):
    """The whole skewed batch through split-K (512-token partitions) in longest-first
    order; the longest, the shortest and evenly spaced sequences against the oracle."""
    wl, q, kp, vp = llama70b_layer
    tables, ctx = wl.block_tables.to(DEV), wl.ctx_lens.to(DEV)
    nbytes = ops.decode_workspace_bytes(wl.batch, q.shape[1], q.shape[2], kp.shape[2],
                                        tables.shape[1], 512)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.paged_decode(q, kp, vp, tables, ctx, q.shape[2] ** -0.5, 512, workspace=ws,
                           device_error=err, seq_order=ops.decode_order(ctx))
    assert int(err.item()) == 0
    by_len = torch.argsort(wl.ctx_lens)
    sample = sorted(set(by_len[-3:].tolist() + by_len[:2].tolist() + [0, 100, 255, 300, 511]))
    assert int(wl.ctx_lens[sample].max()) == 32768  # reaches the clipped tail
    for i in sample:  # one at a time: the oracle expands GQA over dense padded keys
        ck, cv, ctables = _compact_pool(wl, [i], kp, vp)
        ref = oracle_decode(q[[i]], ck, cv, ctables, wl.ctx_lens[[i]])
        assert_attention_close(out[[i]], ref, f"llama70b split512 seq {i}")
    # and every one of the 512 sequences against the oracle's steps on the GPU in fp32
    ref_all = oracle_decode_on_device(q, kp, vp, wl.block_tables, wl.ctx_lens)
    assert_attention_close(out, ref_all, "llama70b split512 every sequence")


def test_llama70b_split_and_unsplit_agree_and_fused_append(llama70b_layer):
    """Split-K and one CTA per (sequence, KV head) agree over the whole batch; the
    fused decode-step append writes exactly what the separate append writes."""
    wl, q, kp, vp = llama70b_layer
    tables, ctx = wl.block_tables.to(DEV), wl.ctx_lens.to(DEV)
    scale = q.shape[2] ** -0.5
    a = _decode(q, kp, vp, tables, ctx, 0).float()
    b = _decode(q, kp, vp, tables, ctx, 512).float()
    assert_attention_close(b, a, "70b split vs unsplit")

    bs = wl.spec.block_size
    pos = wl.ctx_lens.long() - 1
    slots = (wl.block_tables.long().gather(1, (pos // bs).view(-1, 1)).view(-1) * bs
             + pos % bs).to(DEV)
    gen = torch.Generator(device=DEV).manual_seed(2)
    kn = torch.empty((wl.batch, wl.spec.num_kv_heads, wl.spec.head_dim), dtype=torch.bfloat16,
                     device=DEV).normal_(0.0, 0.5, generator=gen)
    vn = torch.empty_like(kn).normal_(0.0, 0.5, generator=gen)
    nbytes = ops.decode_workspace_bytes(wl.batch, q.shape[1], q.shape[2], bs, tables.shape[1], 512)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    ref_k, ref_v = kp.clone(), vp.clone()
    ops.cache_append(ref_k, ref_v, kn, vn, slots)
    want = ops.paged_decode(q, ref_k, ref_v, tables, ctx, scale, 512, workspace=ws)
    del ref_k, ref_v
    got_k, got_v = kp.clone(), vp.clone()
    got = ops.paged_decode_append(q, kn, vn, slots, got_k, got_v, tables, ctx, scale, 512,
                                  workspace=ws)
    assert torch.equal(got, want)
    flat_k = got_k.view(-1, bs, wl.spec.head_dim)  # rows of (block, head)
    heads = wl.spec.num_kv_heads
    row = (slots // bs).view(-1, 1) * heads + torch.arange(heads, device=DEV).view(1, -1)
    assert torch.equal(flat_k[row.view(-1), (slots % bs).repeat_interleave(heads)],
                       kn.view(-1, wl.spec.head_dim))
    flat_v = got_v.view(-1, bs, wl.spec.head_dim)
    assert torch.equal(flat_v[row.view(-1), (slots % bs).repeat_interleave(heads)],
                       vn.view(-1, wl.spec.head_dim))


@pytest.mark.parametrize("split", [64, 512])
def test_planned_step_equals_per_layer_planning(split):
    """A split-K step planned once (ps_paged_decode_plan) and run layer after
    layer with ps_paged_decode_append_planned (the combine re-arms the claim
    counter between layers) gives the same outputs and pool writes, bit for
    bit, as planning inside every layer's call."""
    hq, hkv, d, bs, layers = 32, 8, 128, 16, 3
    lens = [1, 700, 2300, 64, 4000, 33, 512, 513]
    b = len(lens)
    nb = sum((n + bs - 1) // bs for n in lens) + 5
    gen = torch.Generator(device=DEV).manual_seed(9)
    pools = [(torch.randn((nb, hkv, bs, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
             for _ in range(2 * layers)]
    tables = random_tables(lens, bs, nb, seed=9, width=256).to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    pos = ctx.long() - 1
    slots = (tables.long().gather(1, (pos // bs).view(-1, 1)).view(-1) * bs + pos % bs)
    q = (torch.randn((layers, b, hq, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    kn = (torch.randn((layers, b, hkv, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    vn = (torch.randn((layers, b, hkv, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    order = ops.decode_order(ctx)
    nbytes = ops.decode_workspace_bytes(b, hq, d, bs, tables.shape[1], split)
    outs = {}
    for planned in (False, True):
        kp = [p.clone() for p in pools[:layers]]
        vp = [p.clone() for p in pools[layers:]]
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        if planned:
            ops.decode_plan(ctx, ws, hq, d, bs, tables.shape[1], split, seq_order=order)
        res = []
        for layer in range(layers):
            res.append(ops.paged_decode_append(
                q[layer], kn[layer], vn[layer], slots, kp[layer], vp[layer], tables, ctx,
                d**-0.5, split, workspace=ws, device_error=err, seq_order=order,
                planned=planned))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs[planned] = (res, kp, vp)
    for layer in range(layers):
        assert torch.equal(outs[True][0][layer], outs[False][0][layer])
        assert torch.equal(outs[True][1][layer], outs[False][1][layer])
        assert torch.equal(outs[True][2][layer], outs[False][2][layer])
    want = oracle_decode(q[0], outs[True][1][0], outs[True][2][0], tables.cpu(), ctx.cpu())
    assert_attention_close(outs[True][0][0], want, f"planned split {split} vs oracle")
