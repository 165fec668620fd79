"""GPU parity: KV append, append with fused RoPE, and block copy are bit-exact."""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_append, oracle_copy_blocks
from paged_serve_b200 import _lib, ops
from paged_serve_b200.rope import cos_sin_table
from paged_serve_b200.workloads import append_workload
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _slots(num_tokens: int, num_slots: int, seed: int, pad_every: int = 0) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    s = torch.randperm(num_slots, generator=gen)[:num_tokens].to(torch.int64)
    if pad_every:
        s[::pad_every] = -1
    return s


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128])
def test_append_bit_exact(dtype, d):
    t, hkv, bs, nb = 1000, 4, 16, 100
    gen = torch.Generator(device=DEV).manual_seed(0)
    k_pool = torch.randn((nb, hkv, bs, d), generator=gen, device=DEV).to(dtype)
    v_pool = torch.randn((nb, hkv, bs, d), generator=gen, device=DEV).to(dtype)
    key = torch.randn((t, hkv, d), generator=gen, device=DEV).to(dtype)
    value = torch.randn((t, hkv, d), generator=gen, device=DEV).to(dtype)
    slots = _slots(t, nb * bs, 1, pad_every=7)
    ek, ev = oracle_append(k_pool, v_pool, key, value, slots)
    ops.cache_append(k_pool, v_pool, key, value, slots.to(DEV))
    assert torch.equal(k_pool.cpu(), ek) and torch.equal(v_pool.cpu(), ev)


def test_append_from_fused_projection_view():
    """K/V as strided views of one [T, (Hq+2Hkv)*D] projection output."""
    t, hq, hkv, d, bs, nb = 300, 8, 2, 128, 16, 40
    buf = torch.randn((t, (hq + 2 * hkv) * d), device=DEV).to(torch.bfloat16)
    key = buf[:, hq * d : (hq + hkv) * d].view(t, hkv, d)
    value = buf[:, (hq + hkv) * d :].view(t, hkv, d)
    assert key.stride(0) == (hq + 2 * hkv) * d
    k_pool = torch.zeros((nb, hkv, bs, d), dtype=torch.bfloat16, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    slots = _slots(t, nb * bs, 2)
    ek, ev = oracle_append(k_pool, v_pool, key, value, slots)
    ops.cache_append(k_pool, v_pool, key, value, slots.to(DEV))
    assert torch.equal(k_pool.cpu(), ek) and torch.equal(v_pool.cpu(), ev)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d,theta", [(128, 500000.0), (64, 10000.0)])
def test_append_rope_bit_exact_vs_oracle(dtype, d, theta):
    t, hkv, bs, nb, max_pos = 2000, 8, 16, 200, 32768
    gen = torch.Generator(device=DEV).manual_seed(3)
    k_pool = torch.zeros((nb, hkv, bs, d), dtype=dtype, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    key = torch.randn((t, hkv, d), generator=gen, device=DEV).to(dtype)
    value = torch.randn((t, hkv, d), generator=gen, device=DEV).to(dtype)
    slots = _slots(t, nb * bs, 4, pad_every=11)
    pos = torch.randint(0, max_pos, (t,), generator=torch.Generator().manual_seed(5))
    table = cos_sin_table(d, theta, max_pos, dtype, DEV)
    ek, ev = oracle_append(k_pool, v_pool, key, value, slots, pos, table)
    ops.cache_append_rope(k_pool, v_pool, key, value, slots.to(DEV), pos.to(DEV), table)
    assert torch.equal(k_pool.cpu(), ek) and torch.equal(v_pool.cpu(), ev)


@pytest.mark.parametrize("name", ["rope_bf16", "rope_f16"])
def test_append_rope_matches_reference_golden(name):
    """With the reference's own cos/sin rows, the kernel reproduces apply_rotary exactly."""
    g = load_golden(name)
    key = g["key"].to(DEV)
    t, hkv, d = key.shape
    table = torch.cat((g["cos"][:, : d // 2], g["sin"][:, : d // 2]), dim=-1).to(DEV)
    nb = (t + 15) // 16
    k_pool = torch.zeros((nb, hkv, 16, d), dtype=key.dtype, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    slots = torch.arange(t, dtype=torch.int64, device=DEV)
    ops.cache_append_rope(k_pool, v_pool, key, key, slots, slots.clone(), table)
    got = k_pool.permute(0, 2, 1, 3).reshape(nb * 16, hkv, d)[:t].cpu()
    assert torch.equal(got, g["expected"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rope_table_on_device_is_the_reference_formula(dtype):
    """The table equals RotaryEmbedding's cos/sin computed on this device (layers.py:112-116)."""
    d, theta, n = 128, 500000.0, 40000
    table = cos_sin_table(d, theta, n, dtype, DEV)
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=DEV) / d))
    pos = torch.arange(n, device=DEV).view(1, -1)
    freqs = pos.float().unsqueeze(-1) * inv_freq.view(1, 1, -1)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(dtype)[0], emb.sin().to(dtype)[0]
    assert torch.equal(table[:, : d // 2], cos[:, : d // 2])
    assert torch.equal(table[:, d // 2 :], sin[:, : d // 2])
    assert torch.equal(cos[:, : d // 2], cos[:, d // 2 :])


def test_append_rope_full_append_workload_one_layer():
    """The full 16640-token append (256 decode + 8 x 2048 prefill) of one layer."""
    wl = append_workload(seed=0)
    dtype = torch.bfloat16
    gen = torch.Generator(device=DEV).manual_seed(7)
    shape = (wl.num_tokens, wl.num_kv_heads, wl.head_dim)
    key = torch.randn(shape, generator=gen, device=DEV).to(dtype)
    value = torch.randn(shape, generator=gen, device=DEV).to(dtype)
    pshape = (wl.num_blocks, wl.num_kv_heads, wl.block_size, wl.head_dim)
    k_pool = torch.zeros(pshape, dtype=dtype, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    table = cos_sin_table(wl.head_dim, wl.rope_theta, 4096, dtype, DEV)
    ek, ev = oracle_append(k_pool, v_pool, key, value, wl.slot_mapping, wl.positions, table)
    ops.cache_append_rope(k_pool, v_pool, key, value, wl.slot_mapping.to(DEV),
                          wl.positions.to(DEV), table)
    assert torch.equal(k_pool.cpu(), ek) and torch.equal(v_pool.cpu(), ev)


@pytest.mark.parametrize("layers", [1, 3])
def test_copy_blocks_bit_exact(layers):
    nb, hkv, bs, d = 64, 8, 16, 128
    gen = torch.Generator(device=DEV).manual_seed(11)
    shape = (layers, nb, hkv, bs, d) if layers > 1 else (nb, hkv, bs, d)
    k = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
    v = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
    pairs = torch.tensor([[3, 40], [62, 7], [5, 63], [0, 1]], dtype=torch.int64)
    ek, ev = oracle_copy_blocks(k, v, pairs)
    ops.copy_blocks(k, v, pairs.to(DEV))
    assert torch.equal(k.cpu(), ek) and torch.equal(v.cpu(), ev)


@pytest.mark.parametrize("pairs", [[[3, 40], [40, 7]], [[3, 40], [5, 40]], [[40, 7], [3, 40]]])
def test_order_dependent_copy_lists_are_flagged(pairs):
    """A chain or a repeated destination is rejected on the host (check=True) and
    flagged by the kernel (PS_DEVERR_BLOCK_PAIRS); a valid list sets no bit."""
    nb, hkv, bs, d = 64, 8, 16, 128
    k = torch.zeros((nb, hkv, bs, d), dtype=torch.bfloat16, device=DEV)
    v = torch.zeros_like(k)
    bad = torch.tensor(pairs, dtype=torch.int64, device=DEV)
    with pytest.raises(ValueError):
        ops.copy_blocks(k, v, bad, check=True)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.copy_blocks(k, v, bad, err)
    assert int(err.item()) & _lib.PS_DEVERR_BLOCK_PAIRS
    err.zero_()
    ops.copy_blocks(k, v, torch.tensor([[3, 40], [3, 7], [5, 6]], device=DEV), err, check=True)
    assert int(err.item()) == 0


def test_out_of_range_indices_raise_device_error_bits_without_writing():
    """Bad slots/positions/block ids are skipped and reported, never dereferenced."""
    nb, hkv, bs, d = 8, 2, 16, 128
    k_pool = torch.zeros((nb, hkv, bs, d), dtype=torch.bfloat16, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    key = torch.ones((2, hkv, d), dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.cache_append(k_pool, v_pool, key, key,
                     torch.tensor([nb * bs, nb * bs + 100], device=DEV), err)
    assert int(err.item()) & _lib.PS_DEVERR_SLOT
    assert int(k_pool.abs().sum().item()) == 0
    err.zero_()
    table = cos_sin_table(d, 10000.0, 16, torch.bfloat16, DEV)
    ops.cache_append_rope(k_pool, v_pool, key, key, torch.tensor([0, 1], device=DEV),
                          torch.tensor([16, 99], device=DEV), table, err)
    assert int(err.item()) & _lib.PS_DEVERR_POSITION
    assert int(k_pool.abs().sum().item()) == 0
    err.zero_()
    ops.copy_blocks(k_pool, v_pool, torch.tensor([[0, nb]], device=DEV), err)
    assert int(err.item()) & _lib.PS_DEVERR_BLOCK_ID
