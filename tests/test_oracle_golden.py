"""Pins the CPU oracle to the reference's own outputs (fixtures in tests/golden/).

The fixtures were produced by running the reference's ContiguousAttentionBackend,
RotaryEmbedding and apply_rotary (tests/golden/make_golden.py). The oracle
gathers paged KV through block tables and must reproduce them; every GPU
parity test then compares the CUDA kernels against this oracle.
"""

from __future__ import annotations

import pytest
import torch

from oracle import (
    contiguous_attention,
    gather_kv,
    oracle_append,
    oracle_copy_blocks,
    oracle_decode,
    oracle_prefill,
    rope_cos_sin,
    rotate_half,
)
from paged_serve_b200.rope import cos_sin_table
from tests.conftest import load_golden, pool_from_sequences


def _pools(g):
    lens = g["ctx_lens"].tolist() if "ctx_lens" in g else (g["prefix_lens"] + g["q_lens"]).tolist()
    k = pool_from_sequences(g["keys"], lens, g["block_tables"], g["num_blocks"], g["block_size"])
    v = pool_from_sequences(g["values"], lens, g["block_tables"], g["num_blocks"], g["block_size"])
    return k, v


class TestDecodeGolden:
    def test_tiny_paged_equals_contiguous_reference(self):
        """Workload 'tiny' (fp32 host plumbing): paged result == contiguous result."""
        g = load_golden("tiny_decode")
        k, v = _pools(g)
        out = oracle_decode(g["query"], k, v, g["block_tables"], g["ctx_lens"], torch.float32)
        assert torch.allclose(out, g["expected"], atol=1e-6, rtol=0)

    @pytest.mark.parametrize("name", ["decode_bf16_gqa4", "decode_bf16_gqa7"])
    def test_bf16_inputs_fp32_reference(self, name):
        g = load_golden(name)
        k, v = _pools(g)
        out = oracle_decode(g["query"], k, v, g["block_tables"], g["ctx_lens"], torch.float32)
        assert torch.allclose(out, g["expected"], atol=1e-6, rtol=0)

    def test_block_placement_does_not_matter(self):
        """Moving a sequence's blocks elsewhere in the pool changes nothing."""
        g = load_golden("tiny_decode")
        k, v = _pools(g)
        perm = torch.randperm(g["num_blocks"], generator=torch.Generator().manual_seed(9))
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel())
        tables = inv[g["block_tables"].long()].to(torch.int32)
        out = oracle_decode(g["query"], k[perm], v[perm], tables, g["ctx_lens"])
        ref = oracle_decode(g["query"], k, v, g["block_tables"], g["ctx_lens"])
        assert torch.equal(out, ref)

    def test_zero_context_gives_zeros(self):
        g = load_golden("tiny_decode")
        k, v = _pools(g)
        ctx = g["ctx_lens"].clone()
        ctx[1] = 0
        out = oracle_decode(g["query"], k, v, g["block_tables"], ctx)
        assert torch.count_nonzero(out[1]) == 0
        assert torch.allclose(out[0], g["expected"][0], atol=1e-6)


class TestPrefillGolden:
    def test_prefill_prefix_plus_suffix(self):
        g = load_golden("prefill_bf16_gqa4")
        k, v = _pools(g)
        starts = torch.cumsum(g["q_lens"], 0) - g["q_lens"]
        res = oracle_prefill(g["query"], k, v, g["block_tables"], starts.to(torch.int32),
                             g["q_lens"], g["prefix_lens"], torch.float32)
        out = torch.cat([res[i] for i in range(len(res))])
        assert torch.allclose(out, g["expected"], atol=1e-6, rtol=0)


class TestRopeGolden:
    @pytest.mark.parametrize("name,dtype", [("rope_bf16", torch.bfloat16),
                                            ("rope_f16", torch.float16)])
    def test_cos_sin_match_reference(self, name, dtype):
        g = load_golden(name)
        d = g["key"].shape[-1]
        cos, sin = rope_cos_sin(g["positions"], d, g["theta"], dtype)
        assert torch.equal(cos, g["cos"]) and torch.equal(sin, g["sin"])

    @pytest.mark.parametrize("name,dtype", [("rope_bf16", torch.bfloat16),
                                            ("rope_f16", torch.float16)])
    def test_product_table_rows_are_reference_halves(self, name, dtype):
        """cos_sin_table row p = first halves of RotaryEmbedding's cos/sin at p."""
        g = load_golden(name)
        d = g["key"].shape[-1]
        table = cos_sin_table(d, g["theta"], 32768, dtype, "cpu")
        rows = table[g["positions"]]
        assert torch.equal(rows[:, : d // 2], g["cos"][:, : d // 2])
        assert torch.equal(rows[:, d // 2 :], g["sin"][:, : d // 2])
        # and the reference's halves are duplicates (emb = cat(freqs, freqs))
        assert torch.equal(g["cos"][:, : d // 2], g["cos"][:, d // 2 :])

    @pytest.mark.parametrize("name", ["rope_bf16", "rope_f16"])
    def test_append_with_rope_is_bit_exact(self, name):
        g = load_golden(name)
        key = g["key"]
        t, hkv, d = key.shape
        table = torch.cat((g["cos"][:, : d // 2], g["sin"][:, : d // 2]), dim=-1)
        # one slot per token, positions = table rows 0..t-1 (the fixture's own order)
        pool = torch.zeros(((t + 15) // 16, hkv, 16, d), dtype=key.dtype)
        slots = torch.arange(t, dtype=torch.int64)
        kp, _ = oracle_append(pool, pool.clone(), key, key, slots,
                              torch.arange(t, dtype=torch.int64), table)
        got = gather_kv(kp, torch.arange(pool.shape[0], dtype=torch.int32), t)
        assert torch.equal(got, g["expected"])


class TestRopeKnownAnswers:
    """The reference's RoPE known-answer tests, applied to the oracle (tests/test_layers.py)."""

    def test_split_half_convention(self):
        x = torch.tensor([[1.0, 2.0, 3.0, 4.0]])
        assert torch.equal(rotate_half(x), torch.tensor([[-3.0, -4.0, 1.0, 2.0]]))

    def test_four_rotations_are_identity(self):
        x = torch.randn(2, 3, 8)
        assert torch.allclose(rotate_half(rotate_half(rotate_half(rotate_half(x)))), x)

    def test_position_zero_is_identity(self):
        key = torch.randn(3, 2, 8)
        table = cos_sin_table(8, 10000.0, 4, torch.float32, "cpu")
        pool = torch.zeros((1, 2, 16, 8))
        kp, _ = oracle_append(pool, pool.clone(), key, key, torch.arange(3),
                              torch.zeros(3, dtype=torch.int64), table)
        assert torch.allclose(kp[0, :, :3].transpose(0, 1), key, atol=1e-6)

    def test_rotation_preserves_norm(self):
        key = torch.randn(4, 2, 8)
        table = cos_sin_table(8, 10000.0, 16, torch.float32, "cpu")
        pool = torch.zeros((1, 2, 16, 8))
        kp, _ = oracle_append(pool, pool.clone(), key, key, torch.arange(4),
                              torch.arange(4), table)
        rot = kp[0, :, :4].transpose(0, 1)
        assert torch.allclose(rot.norm(dim=-1), key.norm(dim=-1), atol=1e-5)


class TestContiguousMask:
    """Mask semantics of the restated contiguous path (reference tests 89-124)."""

    def test_causal_within_prefill(self):
        q = torch.randn(1, 4, 2, 8)
        k = torch.randn(1, 4, 1, 8)
        v = torch.randn(1, 4, 1, 8)
        out = contiguous_attention(q, k, v, torch.ones(1, 4, dtype=torch.bool), 0)
        # query 0 sees only key 0 -> its output is exactly v0
        assert torch.allclose(out[0, 0, 0], v[0, 0, 0], atol=1e-6)

    def test_padding_does_not_leak(self):
        torch.manual_seed(0)
        q = torch.randn(1, 3, 2, 8)
        k = torch.randn(1, 3, 1, 8)
        v = torch.randn(1, 3, 1, 8)
        alone = contiguous_attention(q, k, v, torch.ones(1, 3, dtype=torch.bool), 0)
        pad = torch.randn(1, 2, 1, 8)
        mask = torch.ones(1, 5, dtype=torch.bool)
        mask[0, :2] = False
        padded = contiguous_attention(torch.cat([torch.randn(1, 2, 2, 8), q], 1),
                                      torch.cat([pad, k], 1), torch.cat([pad, v], 1), mask, 0)
        assert torch.allclose(alone, padded[:, 2:], atol=1e-6)


class TestCopyOracle:
    def test_independent_copies(self):
        k = torch.arange(5 * 2 * 16 * 8, dtype=torch.float32).view(5, 2, 16, 8)
        pairs = torch.tensor([[0, 3], [0, 1], [2, 4]])  # one source may feed several pairs
        kp, vp = oracle_copy_blocks(k, k.clone(), pairs)
        assert torch.equal(kp[3], k[0]) and torch.equal(kp[1], k[0])
        assert torch.equal(kp[4], k[2]) and torch.equal(kp[0], k[0])

    @pytest.mark.parametrize("pairs", [[[0, 3], [3, 1]], [[3, 1], [0, 3]], [[0, 2], [1, 2]]])
    def test_chains_and_repeated_destinations_are_rejected(self, pairs):
        """Pairs run concurrently on the device, so an order-dependent list has no meaning."""
        k = torch.zeros(4, 2, 16, 8)
        with pytest.raises(ValueError):
            oracle_copy_blocks(k, k.clone(), torch.tensor(pairs))

    def test_layered_pools(self):
        k = torch.randn(3, 5, 2, 16, 8)
        kp, _ = oracle_copy_blocks(k, k.clone(), torch.tensor([[1, 4]]))
        assert torch.equal(kp[:, 4], k[:, 1]) and torch.equal(kp[:, 0], k[:, 0])
