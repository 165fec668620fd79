"""GPU: the device slot builder, and continuous batching driven by the block manager.

``ps_build_slot_mapping`` is checked element for element against the slot
formula ``table[p // bs] * bs + p % bs`` (bit-exact, index work). The
continuous-batching replay then drives ``PagedCudaBackend.begin_plan`` with
plans from :class:`BlockManager` — sequences joining mid-flight with
prefix-cache hits, mixed prefill + decode steps, a fork with copy-on-write, a
truncation and frees under a pool smaller than the worst case — and compares
every layer's output with the oracle's contiguous attention over each
sequence's full history; the pool must hold every token's K/V bit-exactly.

A token's K/V is a fixed function of the token ids up to and including it (as a
model's would be), so blocks shared through the prefix cache or copied on
write hold exactly what the borrowing sequence would have computed itself.
"""

from __future__ import annotations

import pytest
import torch

from oracle import contiguous_attention, gather_kv
from paged_serve_b200 import ops
from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.config import ModelConfig
from tests.gpu_util import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
BS = 16


def _expected_slots(tables, ctx, qlens, tq):
    slots, pos = [], []
    for b in range(tables.shape[0]):
        for r in range(tq):
            pad = tq - int(qlens[b])
            if r < pad:
                slots.append(-1)
                pos.append(-1)
            else:
                p = int(ctx[b]) + r - pad
                slots.append(int(tables[b, p // BS]) * BS + p % BS)
                pos.append(p)
    return torch.tensor(slots), torch.tensor(pos)


@pytest.mark.parametrize("tq", [1, 7, 64])
def test_build_slot_mapping_matches_the_formula(tq):
    g = torch.Generator().manual_seed(tq)
    b, width, nb = 37, 40, 4096
    tables = torch.randint(0, nb, (b, width), generator=g, dtype=torch.int32)
    qlens = torch.randint(0, tq + 1, (b,), generator=g, dtype=torch.int32)
    ctx = torch.randint(0, width * BS - tq, (b,), generator=g, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    slots, pos = ops.build_slot_mapping(tables.to(DEV), ctx.to(DEV), qlens.to(DEV), tq, BS, nb,
                                        True, err)
    want_s, want_p = _expected_slots(tables, ctx, qlens, tq)
    assert torch.equal(slots.cpu(), want_s)
    assert torch.equal(pos.cpu(), want_p)
    assert int(err.item()) == 0


def test_build_slot_mapping_flags_bad_inputs():
    tables = torch.tensor([[0, 1], [2, 99], [3, 4]], dtype=torch.int32, device=DEV)
    ctx = torch.tensor([0, 16, 0], dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    # block 99 is outside a 10-block pool
    slots, _ = ops.build_slot_mapping(tables, ctx, torch.tensor([4, 4, 4], dtype=torch.int32,
                                                                device=DEV), 4, BS, 10, True, err)
    assert int(err.item()) == 1  # PS_DEVERR_BLOCK_ID
    assert slots.view(3, 4)[1].tolist() == [-1] * 4
    # a sequence past its table, and q_lens above query_len
    err.zero_()
    ops.build_slot_mapping(tables, torch.tensor([30, 0, 0], dtype=torch.int32, device=DEV),
                           torch.tensor([4, 5, 0], dtype=torch.int32, device=DEV), 4, BS, 10,
                           True, err)
    assert int(err.item()) == 16  # PS_DEVERR_LENGTH


class _History:
    """Token ids per sequence and the K/V a model would produce for them."""

    def __init__(self, model: ModelConfig, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        shape = (model.num_layers, 2, model.num_kv_heads, model.head_dim)
        self.freq = torch.rand(shape, generator=g) * 3.0 + 0.5
        self.phase = torch.rand(shape, generator=g) * 6.283
        self.tokens: dict[int, list[int]] = {}

    def kv(self, layer: int, tokens: list[int], start: int, stop: int):
        h, hs = 0, []
        for t in tokens[:stop]:
            h = (h * 1000003 + t + 1) % (1 << 31)
            hs.append(h / (1 << 31) * 1000.0)
        x = torch.tensor(hs[start:stop], dtype=torch.float64).view(-1, 1, 1)
        k = 0.5 * torch.sin(x * self.freq[layer, 0] + self.phase[layer, 0])
        v = 0.5 * torch.sin(x * self.freq[layer, 1] + self.phase[layer, 1])
        return k.to(torch.bfloat16), v.to(torch.bfloat16)


def _run_step(backend, mgr, hist: _History, seq_ids, model, gen):
    plan = mgr.schedule(seq_ids)
    md = backend.begin_plan(plan)
    b, tq = len(seq_ids), plan.query_len
    hq, hkv, d = model.num_q_heads, model.num_kv_heads, model.head_dim
    for layer in range(model.num_layers):
        q = (torch.randn((b, tq, hq, d), generator=gen) * 0.5).to(torch.bfloat16)
        k = (torch.randn((b, tq, hkv, d), generator=gen) * 0.5).to(torch.bfloat16)  # pads: junk
        v = (torch.randn((b, tq, hkv, d), generator=gen) * 0.5).to(torch.bfloat16)
        for i, sid in enumerate(seq_ids):
            c, n = plan.ctx_before[i], plan.q_lens[i]
            if n:
                k[i, tq - n :], v[i, tq - n :] = hist.kv(layer, hist.tokens[sid], c, c + n)
        out = backend.forward(layer, q.to(DEV), k.to(DEV), v.to(DEV), md).cpu()
        for i, sid in enumerate(seq_ids):
            c, n = plan.ctx_before[i], plan.q_lens[i]
            if not n:
                continue
            kk, vv = hist.kv(layer, hist.tokens[sid], 0, c + n)
            ref = contiguous_attention(q[i : i + 1, tq - n :].float(), kk.float()[None],
                                       vv.float()[None], torch.ones((1, c + n), dtype=torch.bool), c)
            assert_attention_close(out[i, tq - n :], ref[0], f"seq {sid} layer {layer} ctx {c}")
    return plan


@pytest.mark.parametrize("split_mixed", [True, False])
def test_continuous_batching_with_prefix_cache_fork_and_truncate(split_mixed):
    """Mixed steps go through the decode kernel for their one-token sequences
    (split_mixed) or through the prefill kernel for every sequence."""
    model = ModelConfig(name="gqa4", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    backend = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, num_blocks=96,
                               split_tokens=32, debug_invariants=True,
                               split_mixed_steps=split_mixed)
    backend.allocate(num_seq_slots=8, max_seq_len=512)
    mgr = backend.make_block_manager(enable_prefix_caching=True)
    hist = _History(model)
    rng = torch.Generator().manual_seed(1)
    gen = torch.Generator().manual_seed(2)

    def new_tokens(n):
        return torch.randint(0, 50000, (n,), generator=rng).tolist()

    system = new_tokens(40)

    def admit(sid, prompt):
        hist.tokens[sid] = list(prompt)
        mgr.allocate(sid, len(prompt), prompt)

    def decode(sids):
        for sid in sids:
            t = new_tokens(1)
            hist.tokens[sid] += t
            mgr.append_slots(sid, 1, t)

    admit(0, system + new_tokens(30))
    admit(1, new_tokens(45))
    _run_step(backend, mgr, hist, [0, 1], model, gen)
    for _ in range(3):
        decode([0, 1])
        _run_step(backend, mgr, hist, [0, 1], model, gen)
    # a new request shares the system prompt's two full blocks, mixed with decodes
    admit(2, system + new_tokens(21))
    assert mgr.num_computed(2) == 32
    decode([0, 1])
    plan = _run_step(backend, mgr, hist, [0, 1, 2], model, gen)
    assert plan.q_lens == [1, 1, 29]
    # parallel sampling: seq 3 forks seq 0 and writes into the shared partial block
    mgr.fork(0, 3)
    hist.tokens[3] = list(hist.tokens[0])
    decode([0, 1, 2, 3])
    plan = _run_step(backend, mgr, hist, [0, 1, 2, 3], model, gen)
    assert len(plan.copies) == 1
    for _ in range(2):
        decode([0, 1, 2, 3])
        _run_step(backend, mgr, hist, [0, 1, 2, 3], model, gen)
    mgr.free(1)
    del hist.tokens[1]
    # seq 3 rewinds into a shared block (CoW again) and continues with a 9-token chunk
    mgr.truncate_to(3, 50)
    hist.tokens[3] = hist.tokens[3][:50]
    more = new_tokens(9)
    hist.tokens[3] += more
    mgr.append_slots(3, 9, more)
    decode([0, 2])
    plan = _run_step(backend, mgr, hist, [0, 2, 3], model, gen)
    assert plan.copies and plan.q_lens == [1, 1, 9]
    # a request repeating seq 0's whole history so far hits every full block of it
    admit(4, list(hist.tokens[0]) + new_tokens(3))
    assert mgr.num_computed(4) == (len(hist.tokens[0]) // BS) * BS
    for _ in range(2):
        decode([0, 2, 3])
        _run_step(backend, mgr, hist, [0, 2, 3, 4], model, gen)
        decode([4])
    _run_step(backend, mgr, hist, [4], model, gen)
    mgr.check_invariants()
    torch.cuda.synchronize()
    assert int(backend.device_error.item()) == 0
    # every live sequence's K/V sits in the pool bit-exactly, in logical order
    for sid, toks in hist.tokens.items():
        table = torch.tensor(mgr.block_table(sid), dtype=torch.int32)
        for layer in range(model.num_layers):
            kk, vv = hist.kv(layer, toks, 0, len(toks))
            assert torch.equal(gather_kv(backend.k_cache[layer].cpu(), table, len(toks)), kk)
            assert torch.equal(gather_kv(backend.v_cache[layer].cpu(), table, len(toks)), vv)


def test_listed_decode_equals_full_decode_rows_and_leaves_others():
    """ps_paged_decode_listed over a subset, with strided query/out rows (each
    sequence's last row of a [B, query_len] step): listed rows bit-identical to
    the whole-batch decode, unlisted rows untouched; with split-K too."""
    from tests.gpu_util import random_pool, random_tables

    hq, hkv, d, tq = 32, 8, 128, 5
    lens = [1, 700, 2300, 0, 64, 4000, 33]
    b = len(lens)
    nb = sum((n + BS - 1) // BS for n in lens) + 9
    kp, vp = random_pool(nb, hkv, BS, d, torch.bfloat16, DEV, seed=4)
    tables = random_tables(lens, BS, nb, seed=4, width=256).to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(5)
    q = (torch.randn((b, tq, hq, d), generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    listed = torch.tensor([5, 2, 1, 6], dtype=torch.int32, device=DEV)
    for split in (0, 512):
        nbytes = ops.decode_workspace_bytes(b, hq, d, BS, 256, split)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
        full = ops.paged_decode(q[:, tq - 1].contiguous(), kp, vp, tables, ctx, d**-0.5, split,
                                workspace=ws)
        out = torch.full((b, tq, hq, d), 7.0, dtype=torch.bfloat16, device=DEV)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        ops.paged_decode_listed(q[:, tq - 1], kp, vp, tables, ctx, listed, d**-0.5, split,
                                out=out[:, tq - 1], workspace=ws, device_error=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        for i in range(b):
            if i in listed.tolist():
                assert torch.equal(out[i, tq - 1], full[i]), (split, i)
            else:
                assert bool((out[i, tq - 1] == 7.0).all()), (split, i)
        assert bool((out[:, : tq - 1] == 7.0).all())


def test_overlapped_mixed_step_equals_serial_from_any_stream_and_in_a_graph():
    """A mixed step with its decode launch on the side stream (beside the
    prefill) gives the bits of the serial step: from the default stream, from
    another current stream, and replayed from a CUDA graph."""
    model = ModelConfig(name="gqa4", num_layers=1, num_q_heads=8, num_kv_heads=2, head_dim=128)
    backend = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, num_blocks=320,
                               split_tokens=64)
    backend.allocate(num_seq_slots=8, max_seq_len=1024)
    gen = torch.Generator(device=DEV).manual_seed(11)
    backend.k_cache.normal_(0.0, 0.5, generator=gen)
    backend.v_cache.normal_(0.0, 0.5, generator=gen)
    mgr = backend.make_block_manager()
    lens = [300, 517, 64, 900, 33, 700]
    ids = list(range(len(lens)))
    for sid, n in enumerate(lens):
        mgr.allocate(sid, n)
    mgr.schedule(ids)  # the prompts: their K/V is the pool's random contents
    for sid in ids[:4]:
        mgr.append_slots(sid, 1)
    mgr.append_slots(4, 40)  # two prompts add chunks beside four decodes
    mgr.append_slots(5, 7)
    plan = mgr.schedule(ids)
    assert plan.q_lens == [1, 1, 1, 1, 40, 7]
    md = backend.begin_plan(plan)
    assert md.decode_list is not None and md.num_prefill_seqs == 2
    b, tq = len(ids), plan.query_len
    g = torch.Generator(device=DEV).manual_seed(12)
    q = torch.empty((b, tq, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(0, 0.5, generator=g)
    k = torch.empty((b, tq, 2, 128), dtype=torch.bfloat16, device=DEV).normal_(0, 0.5, generator=g)
    v = torch.empty_like(k).normal_(0, 0.5, generator=g)
    rows = [(i, tq - n) for i, n in enumerate(plan.q_lens)]  # (sequence, first new row)

    def run():
        return backend.forward(0, q, k, v, md)  # appends the same K/V to the same slots

    backend.overlap_mixed_steps = False
    serial = run()
    backend.overlap_mixed_steps = True
    over = run()
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        other = run()
    torch.cuda.current_stream(DEV).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = run()
    graph.replay()
    torch.cuda.synchronize()
    assert int(backend.device_error.item()) == 0
    for name, got in (("overlapped", over), ("other stream", other), ("graph", captured)):
        for i, r0 in rows:
            assert torch.equal(got[i, r0:], serial[i, r0:]), (name, i)


def test_long_prompt_chunk_is_split_across_sms_and_matches_the_oracle():
    """A prefill step of one prompt's 300-token chunk over 6000 cached tokens has
    10 work items; begin_plan picks split-K pieces for it, and forward's result
    agrees with the oracle and with the unsplit kernel."""
    from oracle import oracle_prefill

    model = ModelConfig(name="gqa4", num_layers=1, num_q_heads=8, num_kv_heads=2, head_dim=128)
    results = {}
    for split in (True, False):
        backend = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, num_blocks=420,
                                   split_prefill=split)
        backend.allocate(num_seq_slots=1, max_seq_len=8192)
        gen = torch.Generator(device=DEV).manual_seed(21)
        backend.k_cache.normal_(0.0, 0.5, generator=gen)
        backend.v_cache.normal_(0.0, 0.5, generator=gen)
        mgr = backend.make_block_manager()
        mgr.allocate(0, 6000)
        mgr.schedule([0])  # the prompt's first 6000 tokens: the pool's random contents
        mgr.append_slots(0, 300)
        plan = mgr.schedule([0])
        assert plan.q_lens == [300]
        md = backend.begin_plan(plan)
        assert (md.prefill_split_keys > 0) == split
        g = torch.Generator(device=DEV).manual_seed(22)
        q = torch.empty((1, 300, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(
            0, 0.5, generator=g)
        k = torch.empty((1, 300, 2, 128), dtype=torch.bfloat16, device=DEV).normal_(
            0, 0.5, generator=g)
        v = torch.empty_like(k).normal_(0, 0.5, generator=g)
        out = backend.forward(0, q, k, v, md)
        torch.cuda.synchronize()
        assert int(backend.device_error.item()) == 0
        results[split] = out[0].float().cpu()
        if split:
            ref = oracle_prefill(q.reshape(300, 8, 128), backend.k_cache[0], backend.v_cache[0],
                                 md.block_tables.cpu(), md.q_starts.cpu(), md.q_lens.cpu(),
                                 md.ctx_before.cpu(), seqs=[0])
            assert_attention_close(out[0], ref[0], "split long-prompt chunk")
        backend.free()
    assert_attention_close(results[True], results[False], "split vs whole")
