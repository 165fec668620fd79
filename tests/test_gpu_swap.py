"""GPU: swapping KV blocks between the HBM pool and pinned host memory.

``ps_swap_blocks`` must move blocks bit-exactly in both directions for every
layer and both K and V, with any block ids on either side, any grid cap, and
pairs held on the device or in pinned host memory; bad ids set an error bit
and are skipped; pageable host memory is refused before any launch. The
preemption replay swaps a sequence out while others keep running (and reuse
its HBM blocks), brings it back, and checks attention against the oracle and
the pool bit-exactly.
"""

from __future__ import annotations

import pytest
import torch

from paged_serve_b200 import _lib, ops
from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.config import ModelConfig
from tests.test_gpu_block_manager import BS, _History, _run_step

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _pools(layers, blocks, seed, device, pinned=False):
    g = torch.Generator().manual_seed(seed)
    shape = (layers, blocks, 8, BS, 128)
    k = torch.randn(shape, generator=g).to(torch.bfloat16)
    v = torch.randn(shape, generator=g).to(torch.bfloat16)
    if device == "cpu":
        return (k.pin_memory(), v.pin_memory()) if pinned else (k, v)
    return k.to(device), v.to(device)


@pytest.mark.parametrize("max_ctas", [0, 1, 5])
def test_swap_round_trip_is_bit_exact(max_ctas):
    dk, dv = _pools(3, 40, 0, DEV)
    hk = torch.zeros((3, 24, 8, BS, 128), dtype=torch.bfloat16).pin_memory()
    hv = torch.zeros_like(hk).pin_memory()
    g = torch.Generator().manual_seed(max_ctas)
    src = torch.randperm(40, generator=g)[:17]
    dst = torch.randperm(24, generator=g)[:17]
    out_pairs = torch.stack([src, dst], 1).contiguous().to(DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.swap_blocks(hk, hv, dk, dv, out_pairs, max_ctas, err)
    torch.cuda.synchronize()
    assert torch.equal(hk[:, dst], dk[:, src].cpu()) and torch.equal(hv[:, dst], dv[:, src].cpu())
    # back in, to different HBM blocks; pairs read straight from pinned host memory
    back = torch.randperm(40, generator=g)[:17]
    in_pairs = torch.stack([dst, back], 1).contiguous().pin_memory()
    ek, ev = torch.zeros_like(dk), torch.zeros_like(dv)
    ops.swap_blocks(ek, ev, hk, hv, in_pairs, max_ctas, err)
    torch.cuda.synchronize()
    assert torch.equal(ek[:, back], dk[:, src]) and torch.equal(ev[:, back], dv[:, src])
    untouched = torch.ones(40, dtype=torch.bool)
    untouched[back] = False
    assert not ek[:, untouched].any()
    assert int(err.item()) == 0


def test_swap_flags_bad_ids_and_copies_the_rest():
    dk, dv = _pools(2, 8, 1, DEV)
    hk = torch.zeros((2, 4, 8, BS, 128), dtype=torch.bfloat16).pin_memory()
    hv = torch.zeros_like(hk).pin_memory()
    pairs = torch.tensor([[1, 0], [9, 1], [2, 4], [3, 3]], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.swap_blocks(hk, hv, dk, dv, pairs, 0, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1  # PS_DEVERR_BLOCK_ID
    assert torch.equal(hk[:, 0], dk[:, 1].cpu()) and torch.equal(hk[:, 3], dk[:, 3].cpu())
    assert not hk[:, 1].any() and not hk[:, 2].any()


def test_swap_refuses_pageable_host_memory():
    dk, dv = _pools(1, 4, 2, DEV)
    pk = torch.zeros((1, 4, 8, BS, 128), dtype=torch.bfloat16)  # not pinned
    pv = torch.zeros_like(pk)
    pairs = torch.tensor([[0, 0]], dtype=torch.int64, device=DEV)
    with pytest.raises(ValueError, match="pageable"):
        ops.swap_blocks(pk, pv, dk, dv, pairs)
    # the C ABI checks too, without launching anything
    lib = _lib.load()
    block_bytes = 8 * BS * 128 * 2
    st = lib.ps_swap_blocks(pk.data_ptr(), pv.data_ptr(), 4, 0, dk.data_ptr(), dv.data_ptr(), 4,
                            0, pairs.data_ptr(), 1, 1, block_bytes, 0, None,
                            torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PS_ERR_INVALID
    assert b"pageable" in lib.ps_last_error_string()
    torch.cuda.synchronize()


def test_preemption_by_swap_mid_flight():
    model = ModelConfig(name="gqa4", num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128)
    backend = PagedCudaBackend(model, device=DEV, dtype=torch.bfloat16, num_blocks=24,
                               split_tokens=32, debug_invariants=True)
    backend.allocate(num_seq_slots=4, max_seq_len=256)
    backend.allocate_swap_space(16)
    mgr = backend.make_block_manager()
    hist = _History(model, seed=3)
    rng = torch.Generator().manual_seed(4)
    gen = torch.Generator().manual_seed(5)

    def new_tokens(n):
        return torch.randint(0, 50000, (n,), generator=rng).tolist()

    def admit(sid, n):
        hist.tokens[sid] = new_tokens(n)
        mgr.allocate(sid, n, hist.tokens[sid])

    def decode(sids):
        for sid in sids:
            t = new_tokens(1)
            hist.tokens[sid] += t
            mgr.append_slots(sid, 1, t)

    admit(0, 100)
    admit(1, 120)  # 7 + 8 blocks of 24
    _run_step(backend, mgr, hist, [0, 1], model, gen)
    decode([0, 1])
    _run_step(backend, mgr, hist, [0, 1], model, gen)
    # memory pressure: seq 1 is swapped out, seq 2 takes (and overwrites) its blocks
    freed = set(mgr.block_table(1))
    mgr.swap_out(1)
    admit(2, 140)
    assert freed & set(mgr.block_table(2)), "the new sequence reuses the swapped blocks"
    decode([0])
    plan = _run_step(backend, mgr, hist, [0, 2], model, gen)
    assert len(plan.swap_out) == 8
    for _ in range(3):
        decode([0, 2])
        _run_step(backend, mgr, hist, [0, 2], model, gen)
    mgr.free(2)
    del hist.tokens[2]
    mgr.swap_in(1)
    decode([0, 1])
    plan = _run_step(backend, mgr, hist, [0, 1], model, gen)
    assert len(plan.swap_in) == 8
    for _ in range(2):
        decode([0, 1])
        _run_step(backend, mgr, hist, [0, 1], model, gen)
    torch.cuda.synchronize()
    assert int(backend.device_error.item()) == 0
    from oracle import gather_kv

    for sid, toks in hist.tokens.items():
        table = torch.tensor(mgr.block_table(sid), dtype=torch.int32)
        for layer in range(model.num_layers):
            kk, vv = hist.kv(layer, toks, 0, len(toks))
            assert torch.equal(gather_kv(backend.k_cache[layer].cpu(), table, len(toks)), kk)
            assert torch.equal(gather_kv(backend.v_cache[layer].cpu(), table, len(toks)), vv)
