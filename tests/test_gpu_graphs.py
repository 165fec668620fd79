"""GPU: the decode step's attention loop replayed from a CUDA graph.

The captured graph runs the same kernels with the same launch shapes as the
eager path, so its outputs and pool writes must equal the eager ones
bit-exactly (and the oracle within the attention tolerance). Static metadata is
refilled in place between replays: growing contexts, a changing set of live
sequences from the block manager, and inactive rows that must write nothing
and output zeros.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_decode
from paged_serve_b200 import ops
from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.config import ModelConfig
from paged_serve_b200.graphs import DecodeGraph
from tests.gpu_util import assert_attention_close, random_tables
from tests.test_gpu_block_manager import _History, _run_step

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MODEL = ModelConfig(name="gqa4", num_layers=3, num_q_heads=8, num_kv_heads=2, head_dim=128)


def _backend(num_blocks=256, split=64, slots=8, max_len=1024):
    be = PagedCudaBackend(MODEL, device=DEV, dtype=torch.bfloat16, num_blocks=num_blocks,
                          split_tokens=split)
    be.allocate(num_seq_slots=slots, max_seq_len=max_len)
    g = torch.Generator(device=DEV).manual_seed(0)
    be.k_cache.normal_(0, 0.5, generator=g)
    be.v_cache.normal_(0, 0.5, generator=g)
    return be


@pytest.mark.parametrize("split", [0, 64])
def test_graph_replay_matches_eager_bit_exactly(split):
    be = _backend(split=split)
    lens = [37, 300, 1, 129, 512, 64]
    tables = random_tables([n + 2 for n in lens], 16, be.num_blocks, seed=1, width=34)
    graph = DecodeGraph(be, batch=8)
    gen = torch.Generator(device=DEV).manual_seed(2)
    ref_k, ref_v = be.k_cache.clone(), be.v_cache.clone()
    for step in range(2):  # contexts grow by one token per step
        ctx = torch.tensor([n + step for n in lens], dtype=torch.int32)
        for t in (graph.query, graph.key, graph.value):
            t.normal_(0, 0.5, generator=gen)
        graph.load(tables, ctx)
        outs = graph.replay()
        # eager: the same kernels on copies of the pools
        pos = ctx.long() - 1
        slots = (tables.long().gather(1, (pos // 16).view(-1, 1)).view(-1) * 16 + pos % 16)
        n = len(lens)
        for layer in range(MODEL.num_layers):
            ops.cache_append(ref_k[layer], ref_v[layer], graph.key[layer, :n, 0],
                             graph.value[layer, :n, 0], slots.to(DEV))
            want = ops.paged_decode(graph.query[layer, :n, 0], ref_k[layer], ref_v[layer],
                                    tables.to(DEV), ctx.to(DEV), be.scale, split,
                                    workspace=be._workspace)
            got = outs[layer][:, 0]
            assert torch.equal(got[:n], want), f"layer {layer} step {step}"
            assert not got[n:].any(), "inactive rows output zeros"
            ref = oracle_decode(graph.query[layer, :n, 0], ref_k[layer], ref_v[layer], tables,
                                ctx)
            assert_attention_close(got[:n], ref, f"layer {layer} step {step}")
        torch.cuda.synchronize()
        assert torch.equal(be.k_cache, ref_k) and torch.equal(be.v_cache, ref_v)


def test_graph_with_block_manager_and_changing_batch():
    be = _backend(num_blocks=64, split=32, slots=4, max_len=512)
    mgr = be.make_block_manager()
    hist = _History(MODEL, seed=7)
    rng = torch.Generator().manual_seed(8)
    gen = torch.Generator().manual_seed(9)
    graph = DecodeGraph(be, batch=4)

    def admit(sid, n):
        hist.tokens[sid] = torch.randint(0, 50000, (n,), generator=rng).tolist()
        mgr.allocate(sid, n, hist.tokens[sid])
        _run_step(be, mgr, hist, [sid], MODEL, gen)  # eager prefill

    def graph_step(sids):
        for sid in sids:
            t = torch.randint(0, 50000, (1,), generator=rng).tolist()
            hist.tokens[sid] += t
            mgr.append_slots(sid, 1, t)
        plan = mgr.schedule(sids)
        for layer in range(MODEL.num_layers):
            graph.query[layer].normal_(0, 0.5, generator=torch.Generator(device=DEV).manual_seed(
                layer + 100 * len(hist.tokens[sids[0]])))
            for i, sid in enumerate(sids):
                k, v = hist.kv(layer, hist.tokens[sid], plan.ctx_before[i], plan.seq_lens[i])
                graph.key[layer, i] = k.to(DEV)
                graph.value[layer, i] = v.to(DEV)
        graph.load_plan(plan)
        outs = graph.replay()
        for layer in range(MODEL.num_layers):
            for i, sid in enumerate(sids):
                kk, vv = hist.kv(layer, hist.tokens[sid], 0, plan.seq_lens[i])
                q = graph.query[layer, i : i + 1, 0].cpu()
                from oracle import contiguous_attention

                ref = contiguous_attention(q.float()[:, None], kk.float()[None], vv.float()[None],
                                           torch.ones((1, plan.seq_lens[i]), dtype=torch.bool),
                                           plan.seq_lens[i] - 1)
                assert_attention_close(outs[layer][i, 0], ref[0, 0], f"seq {sid} layer {layer}")
            assert not outs[layer][len(sids):].any()

    admit(0, 70)
    admit(1, 33)
    for _ in range(3):
        graph_step([0, 1])
    admit(2, 100)
    for _ in range(2):
        graph_step([2, 0, 1])  # a new row order: tables are reloaded, not assumed
    mgr.free(0)
    del hist.tokens[0]
    for _ in range(2):
        graph_step([1, 2])
    torch.cuda.synchronize()
    assert int(be.device_error.item()) == 0


@pytest.mark.parametrize("split", [0, 16])
def test_back_to_back_dependent_launches_keep_stream_order(split):
    """The append, copy, decode and prefill kernels launch with programmatic
    stream serialization, so each may begin while the one before it drains.
    A chain in which every launch reads what the previous one wrote — append
    rows into a block, copy that block, decode and prefill over the copy, then
    overwrite the source — must give the oracle's answer eagerly and from a
    captured graph, and the two runs must agree bit for bit."""
    from oracle import oracle_append, oracle_copy_blocks, oracle_prefill
    from paged_serve_b200.rope import cos_sin_table

    hq, hkv, d, bs, nb = 8, 2, 128, 16, 64
    gen = torch.Generator(device=DEV).manual_seed(7)
    k0 = (torch.randn((nb, hkv, bs, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    v0 = (torch.randn((nb, hkv, bs, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    key = (torch.randn((bs, hkv, d), generator=gen, device=DEV)).to(torch.bfloat16)
    val = (torch.randn((bs, hkv, d), generator=gen, device=DEV)).to(torch.bfloat16)
    key2 = (torch.randn((bs, hkv, d), generator=gen, device=DEV)).to(torch.bfloat16)
    q = (torch.randn((1, hq, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    qp = (torch.randn((bs, hq, d), generator=gen, device=DEV) * 0.5).to(torch.bfloat16)
    src, dst = 5, 40
    slots = (torch.arange(bs) + src * bs).to(DEV)
    pos = torch.arange(100, 100 + bs).to(DEV)
    table = cos_sin_table(d, 10000.0, 256, torch.bfloat16, DEV)
    pairs = torch.tensor([[src, dst]], dtype=torch.int64, device=DEV)
    bt = torch.tensor([[3, dst]], dtype=torch.int32, device=DEV)  # 32 keys: block 3, then the copy
    ctx = torch.tensor([2 * bs], dtype=torch.int32, device=DEV)
    nbytes = ops.decode_workspace_bytes(1, hq, d, bs, 2, split)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
    qs = torch.tensor([0], dtype=torch.int32, device=DEV)
    ql = torch.tensor([bs], dtype=torch.int32, device=DEV)
    cl = torch.tensor([bs], dtype=torch.int32, device=DEV)

    def chain(kp, vp, out, out_p):
        ops.cache_append_rope(kp, vp, key, val, slots, pos, table)
        ops.copy_blocks(kp, vp, pairs)
        ops.paged_decode(q, kp, vp, bt, ctx, d**-0.5, split, out=out, workspace=ws)
        ops.paged_prefill(qp, kp, vp, bt, qs, ql, cl, bs, d**-0.5, out=out_p)
        ops.cache_append(kp, vp, key2, val, slots)  # overwrite the source block afterwards

    kp, vp = k0.clone(), v0.clone()
    out, out_p = torch.empty_like(q), torch.empty_like(qp)
    chain(kp, vp, out, out_p)
    torch.cuda.synchronize()
    # oracle: the same chain on the CPU
    ek, ev = oracle_append(k0, v0, key, val, slots, pos, table)
    ek, ev = oracle_copy_blocks(ek, ev, pairs.cpu())
    want = oracle_decode(q, ek, ev, bt.cpu(), ctx.cpu())
    want_p = oracle_prefill(qp, ek, ev, bt.cpu(), qs.cpu(), ql.cpu(), cl.cpu())[0]
    ek, ev = oracle_append(ek, ev, key2, val, slots)
    assert_attention_close(out, want, "decode after append + copy")
    assert_attention_close(out_p, want_p, "prefill after append + copy")
    assert torch.equal(kp.cpu(), ek) and torch.equal(vp.cpu(), ev)

    # the same chain captured once and replayed
    gk, gv = k0.clone(), v0.clone()
    g_out, g_out_p = torch.empty_like(q), torch.empty_like(qp)
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        chain(gk.clone(), gv.clone(), g_out.clone(), g_out_p.clone())  # warm-up off the graph
    torch.cuda.current_stream(DEV).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain(gk, gv, g_out, g_out_p)
    gk.copy_(k0)
    gv.copy_(v0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(g_out, out) and torch.equal(g_out_p, out_p)
    assert torch.equal(gk, kp) and torch.equal(gv, vp)
