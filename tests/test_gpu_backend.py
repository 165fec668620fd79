"""GPU parity of PagedCudaBackend against the contiguous path, step by step.

Replays what the reference's static-batching engine does (pagedserve/engine.py:
left-padded prefill, then one decode step per token with padding_mask grown by
one column) and compares every layer's output with the restated contiguous
backend on the same dense, left-padded history; the paged pool must hold every
real token bit-exactly in logical order.
"""

from __future__ import annotations

import pytest
import torch

from oracle import contiguous_attention, gather_kv
from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.config import ModelConfig
from paged_serve_b200.interface import StepInput
from tests.gpu_util import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _run_engine(backend: PagedCudaBackend, model: ModelConfig, prompt_lens, decode_steps,
                use_tables: bool, seed: int = 0):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    b = len(prompt_lens)
    max_prompt = max(prompt_lens)
    total = max_prompt + decode_steps
    hq, hkv, d, nl = model.num_q_heads, model.num_kv_heads, model.head_dim, model.num_layers
    backend.allocate(num_seq_slots=b, max_seq_len=total)
    mask = torch.zeros((b, total), dtype=torch.bool)
    for i, n in enumerate(prompt_lens):
        mask[i, max_prompt - n : max_prompt] = True
    k_hist = torch.zeros((nl, b, total, hkv, d))
    v_hist = torch.zeros_like(k_hist)
    seq_lens = torch.tensor(prompt_lens, dtype=torch.int32)
    # engine-managed pages: a shuffled assignment of the pool to sequences
    bsz = backend.block_size
    width = (total + bsz - 1) // bsz
    perm = torch.randperm(backend.num_blocks, generator=torch.Generator().manual_seed(seed))
    tables = perm[: b * width].view(b, width).to(torch.int32)

    def slots_for(ctx, tq):
        """Flat slots of this step's tokens under left padding (-1 for pads)."""
        real = mask[:, ctx : ctx + tq]
        before = mask[:, :ctx].sum(1, keepdim=True)
        logical = before + real.cumsum(1) - 1
        blk = tables.long().gather(1, (logical.clamp(min=0) // bsz))
        return torch.where(real, blk * bsz + logical % bsz, -1).reshape(-1)

    steps = [(0, max_prompt)] + [(max_prompt + s, 1) for s in range(decode_steps)]
    for ctx, tq in steps:
        if tq == 1:
            mask[:, ctx] = True
            seq_lens = seq_lens + 1
        step = StepInput(
            query_len=tq, context_len=ctx, seq_lens=seq_lens.to(DEV),
            padding_mask=mask[:, : ctx + tq].to(DEV), is_prefill=tq > 1,
            block_tables=tables.to(DEV) if use_tables else None,
            slot_mapping=slots_for(ctx, tq).to(DEV) if use_tables else None,
        )
        md = backend.begin_step(step)
        for layer in range(nl):
            q = (torch.randn((b, tq, hq, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
            k = (torch.randn((b, tq, hkv, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
            v = (torch.randn((b, tq, hkv, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
            out = backend.forward(layer, q, k, v, md)
            k_hist[layer, :, ctx : ctx + tq] = k.float().cpu()
            v_hist[layer, :, ctx : ctx + tq] = v.float().cpu()
            ref = contiguous_attention(q.float().cpu(), k_hist[layer, :, : ctx + tq],
                                       v_hist[layer, :, : ctx + tq], mask[:, : ctx + tq], ctx)
            real = mask[:, ctx : ctx + tq]
            assert_attention_close(out.cpu()[real], ref[real], f"layer {layer} ctx {ctx}")
    torch.cuda.synchronize()
    # the pool holds every real token, in logical order, bit-exactly
    for layer in range(nl):
        for i in range(b):
            n = int(mask[i].sum())
            row = tables[i] if use_tables else backend._identity_tables[i].cpu()
            got_k = gather_kv(backend.k_cache[layer].cpu(), row, n).float()
            assert torch.equal(got_k, k_hist[layer, i][mask[i]])
            got_v = gather_kv(backend.v_cache[layer].cpu(), row, n).float()
            assert torch.equal(got_v, v_hist[layer, i][mask[i]])
    return seq_lens


@pytest.mark.parametrize("use_tables", [False, True])
@pytest.mark.parametrize("split", [0, 16])
def test_static_engine_replay(use_tables, split):
    model = ModelConfig("tiny-gqa4", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    be = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, split_tokens=split,
                          num_blocks=64 if use_tables else None, debug_invariants=True)
    seq_lens = _run_engine(be, model, [5, 37, 3, 20], decode_steps=6, use_tables=use_tables)
    stats = be.memory_stats()
    per_token = 2 * model.num_layers * model.num_kv_heads * model.head_dim * 2
    assert stats.live_bytes == int(seq_lens.sum()) * per_token
    assert stats.allocated_bytes == 2 * be.k_cache.numel() * 2


@pytest.mark.parametrize("use_tables", [False, True])
def test_qwen_geometry_prefill_and_decode_replay(use_tables):
    """Head dim 64 with 7 query heads per KV head (the reference's default model,
    Qwen2.5-0.5B): a left-padded prefill of uneven prompts, then decode steps."""
    model = ModelConfig("qwen-like", num_layers=2, num_q_heads=14, num_kv_heads=2, head_dim=64)
    be = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, split_tokens=32)
    _run_engine(be, model, [37, 5, 130], decode_steps=12, use_tables=use_tables)


@pytest.mark.parametrize("block_size", [8, 32])
def test_static_engine_replay_other_block_sizes(block_size):
    """CacheConfig.block_size is a knob the reference sweeps: prefill + decode at 8 and 32."""
    model = ModelConfig("tiny", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    be = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, block_size=block_size,
                          split_tokens=64)
    _run_engine(be, model, [37, 5, 130], decode_steps=6, use_tables=False)
    be2 = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, block_size=block_size,
                           split_tokens=64)
    _run_engine(be2, model, [20, 64, 3], decode_steps=4, use_tables=True)


@pytest.mark.parametrize("use_tables", [False, True])
def test_static_engine_long_prompt_prefill_splits_the_key_range(use_tables):
    """A left-padded prefill of a 1,500-token prompt next to a 700-token one has
    96 work items on 148 SMs: begin_step picks split-K pieces of the key range
    (ps_paged_prefill_split), and every layer still matches the contiguous path."""
    model = ModelConfig("tiny-gqa4", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    be = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16,
                          num_blocks=256 if use_tables else None)
    seen = []
    begin = be.begin_step

    def spy(step):
        md = begin(step)
        seen.append(md.prefill_split_keys)
        return md

    be.begin_step = spy
    _run_engine(be, model, [1500, 700], decode_steps=2, use_tables=use_tables)
    assert seen[0] > 0 and seen[1:] == [0, 0]  # the prefill split; decode steps never do


def test_decode_forward_allocates_nothing():
    """The decode loop reserves everything up front (the reference's rule, AGENTS.md 2.5):
    a query_len-1 forward returns a view of the per-layer buffer and allocates nothing."""
    model = ModelConfig("tiny", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    be = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, split_tokens=16)
    be.allocate(num_seq_slots=4, max_seq_len=64)
    mask = torch.zeros((3, 40), dtype=torch.bool)
    mask[:, 10:] = True
    step = StepInput(query_len=1, context_len=39, seq_lens=torch.full((3,), 30, dtype=torch.int32),
                     padding_mask=mask.to(DEV), is_prefill=False)
    md = be.begin_step(step)
    q = torch.randn((3, 1, 8, 128), device=DEV).to(torch.bfloat16)
    k = torch.randn((3, 1, 2, 128), device=DEV).to(torch.bfloat16)
    v = torch.randn_like(k)
    be.forward(1, q, k, v, md)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(DEV)
    out = be.forward(1, q, k, v, md)
    assert torch.cuda.memory_allocated(DEV) == before
    assert out.untyped_storage().data_ptr() == be._decode_out.untyped_storage().data_ptr()
    assert out.shape == (3, 1, 8, 128) and torch.isfinite(out.float()).all()


def test_write_kv_rope_matches_rotated_append():
    """The fused RoPE append equals rotating K on the host side and appending."""
    from paged_serve_b200.rope import cos_sin_table

    model = ModelConfig("rope", num_layers=1, num_q_heads=8, num_kv_heads=2, head_dim=128,
                        rope_theta=500000.0)
    a = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16)
    b = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16)
    a.allocate(2, 64)
    b.allocate(2, 64)
    mask = torch.ones((2, 10), dtype=torch.bool)
    mask[0, :3] = False
    step = StepInput(query_len=10, context_len=0, seq_lens=torch.tensor([7, 10], device=DEV),
                     padding_mask=mask.to(DEV), is_prefill=True)
    ma, mb = a.begin_step(step), b.begin_step(step)
    k = torch.randn((2, 10, 2, 128), device=DEV).to(torch.bfloat16)
    v = torch.randn((2, 10, 2, 128), device=DEV).to(torch.bfloat16)
    a.write_kv_rope(0, k, v, ma)
    table = cos_sin_table(128, 500000.0, 64, torch.bfloat16, DEV)
    pos = mb.positions.clamp(min=0)
    rows = table[pos]
    c, s = rows[:, :64], rows[:, 64:]
    cos = torch.cat((c, c), -1).view(2, 10, 1, 128)
    sin = torch.cat((s, s), -1).view(2, 10, 1, 128)
    rot = (k * cos) + (torch.cat((-k[..., 64:], k[..., :64]), -1) * sin)
    from paged_serve_b200 import ops

    ops.cache_append(b.k_cache[0], b.v_cache[0], rot.view(20, 2, 128), v.view(20, 2, 128),
                     mb.slot_mapping)
    assert torch.equal(a.k_cache, b.k_cache) and torch.equal(a.v_cache, b.v_cache)
