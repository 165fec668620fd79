"""Seeded synthetic workloads for the paged KV hot path.

The reference publishes no dataset for this path (its load generator reads a
ShareGPT-style file that is not part of it), so every benchmark and parity case
draws its inputs from fixed seeds with the shapes of the five workloads below:

* ``tiny``       — 1 layer, Hq 8 / Hkv 2, D 64, ctx {17, 64, 100, 255}, pool 128
                   blocks of 16, fp32 on the host (plumbing check).
* ``llama8b``    — Llama-3-8B decode: 32 layers, Hq 32 / Hkv 8, D 128, bs 16,
                   batch 256, ctx ~ U[512, 4096], pool 1.25x the blocks needed,
                   block ids from a seeded shuffle, values 0.5*N(0,1), scale 1/sqrt(128).
* ``append``     — one append per layer x 32 layers of 256 decode tokens + 8
                   prefill sequences of 2048 tokens (16640 tokens of K/V [., 8, 128]).
* ``prefix``     — prefix-cached prefill: 64 sequences share a 1024-token prefix
                   (64 blocks); each adds 512 new tokens; 8 sequences fork at
                   prefix length 1000, so their partially shared block is copied
                   (copy-on-write) before their suffix is written.
* ``llama70b``   — long-context skewed decode: 80 layers, Hq 64 / Hkv 8, D 128,
                   batch 512, lengths lognormal (median 2048, sigma 1.0) clipped to
                   [128, 32768].

Metadata (lengths, block tables, slots) is built on the host with a CPU
``torch.Generator``; tensor contents are drawn on the target device.
"""

from __future__ import annotations

import heapq
import math
from dataclasses import dataclass

import torch

__all__ = [
    "DecodeSpec",
    "DecodeWorkload",
    "SPECS",
    "AppendWorkload",
    "PrefixWorkload",
    "assign_blocks",
    "decode_workload",
    "append_workload",
    "prefix_workload",
    "lpt_shard",
]


@dataclass(frozen=True)
class DecodeSpec:
    name: str
    num_layers: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    batch: int
    lengths: str  # "uniform" | "lognormal" | "fixed"
    len_lo: int = 0
    len_hi: int = 0
    median: float = 0.0
    sigma: float = 0.0
    fixed: tuple[int, ...] = ()
    pool_factor: float = 1.25
    pool_blocks: int = 0  # explicit pool size (overrides pool_factor)
    value_scale: float = 0.5
    rope_theta: float = 500000.0

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)


SPECS: dict[str, DecodeSpec] = {
    "tiny": DecodeSpec("tiny", 1, 8, 2, 64, 16, 4, "fixed", fixed=(17, 64, 100, 255),
                       pool_blocks=128, value_scale=1.0, rope_theta=10000.0),
    "llama8b": DecodeSpec("llama8b", 32, 32, 8, 128, 16, 256, "uniform", 512, 4096),
    "llama70b": DecodeSpec("llama70b", 80, 64, 8, 128, 16, 512, "lognormal", 128, 32768,
                           median=2048.0, sigma=1.0),
    # The reference's default model (Qwen2.5-0.5B: 24 layers, 14 query heads over 2
    # KV heads, head dim 64) with the 8B workload's batch and lengths.
    "qwen05b": DecodeSpec("qwen05b", 24, 14, 2, 64, 16, 256, "uniform", 512, 4096,
                          rope_theta=1000000.0),
}


def draw_lengths(spec: DecodeSpec, batch: int, gen: torch.Generator) -> torch.Tensor:
    """Context lengths (keys attended, newest token included) as int64 [batch]."""
    if spec.lengths == "fixed":
        return torch.tensor(spec.fixed[:batch], dtype=torch.int64)
    if spec.lengths == "uniform":
        return torch.randint(spec.len_lo, spec.len_hi + 1, (batch,), generator=gen)
    if spec.lengths == "lognormal":
        z = torch.randn(batch, generator=gen, dtype=torch.float64)
        x = torch.exp(math.log(spec.median) + spec.sigma * z)
        return x.round().clamp(spec.len_lo, spec.len_hi).to(torch.int64)
    raise ValueError(spec.lengths)


def lpt_shard(lengths: torch.Tensor, world: int) -> list[torch.Tensor]:
    """Greedy token-balanced (longest-processing-time-first) split of sequences.

    Sorts by length descending and gives each sequence to the rank holding the
    fewest tokens so far (ties to the lower rank). Returns per-rank index
    tensors in ascending order.
    """
    order = torch.argsort(lengths, descending=True, stable=True).tolist()
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    owned: list[list[int]] = [[] for _ in range(world)]
    lens = lengths.tolist()
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    return [torch.tensor(sorted(o), dtype=torch.int64) for o in owned]


def assign_blocks(
    blocks_per_seq: list[int], num_blocks: int, gen: torch.Generator, width: int | None = None
) -> torch.Tensor:
    """Block tables [B, width] int32 from a seeded shuffle of the pool ids.

    Sequences take consecutive runs of one random permutation of
    ``range(num_blocks)``, so no two sequences share a block; unused entries are 0.
    """
    need = sum(blocks_per_seq)
    if need > num_blocks:
        raise ValueError(f"pool of {num_blocks} blocks cannot hold {need}")
    perm = torch.randperm(num_blocks, generator=gen)
    width = width or max(blocks_per_seq + [1])
    tables = torch.zeros((len(blocks_per_seq), width), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(blocks_per_seq):
        tables[i, :n] = perm[pos : pos + n].to(torch.int32)
        pos += n
    return tables


@dataclass
class DecodeWorkload:
    """One rank's decode batch: metadata on the host, ready to move to a device."""

    spec: DecodeSpec
    seq_ids: torch.Tensor  # global sequence ids owned by this rank
    ctx_lens: torch.Tensor  # int32 [B]
    block_tables: torch.Tensor  # int32 [B, max_blocks]
    num_blocks: int
    seed: int

    @property
    def batch(self) -> int:
        return int(self.ctx_lens.shape[0])

    @property
    def total_tokens(self) -> int:
        return int(self.ctx_lens.sum())

    def kv_bytes_per_layer(self, elem: int = 2) -> int:
        s = self.spec
        return self.total_tokens * s.num_kv_heads * s.head_dim * elem * 2

    def algorithmic_bytes_per_layer(self, elem: int = 2) -> int:
        """HBM bytes one decode layer must move: K+V, q read + out write, block ids."""
        s = self.spec
        blocks = int(((self.ctx_lens + s.block_size - 1) // s.block_size).sum())
        return (self.kv_bytes_per_layer(elem) + 2 * self.batch * s.num_q_heads * s.head_dim * elem
                + blocks * 4)

    def flops_per_layer(self) -> int:
        s = self.spec
        return 4 * s.num_q_heads * s.head_dim * self.total_tokens


def decode_workload(
    name: str, seed: int = 0, rank: int = 0, world: int = 1, weak: bool = True,
    batch: int | None = None,
) -> DecodeWorkload:
    """Draw the named decode workload and return rank ``rank``'s share.

    ``weak=True``: the global batch is ``world`` copies of one ``batch``-sequence
    draw (sequence ids ``c * batch + i`` for copy ``c``), so the greedy
    token-balanced split hands every rank the same multiset of lengths: the
    per-GPU work is exactly the one-GPU workload at every world size, and a
    weak-scaling curve measures the system, not the draw. ``weak=False``: the
    global batch is one ``batch``-sequence draw split across the ranks. Either
    way the split is :func:`lpt_shard`. Each rank's pool is ``pool_factor`` x
    its blocks; block ids and tensor contents differ per rank.
    """
    spec = SPECS[name]
    gen = torch.Generator().manual_seed(seed)
    per = batch if batch is not None else spec.batch
    total = per * world if weak else per
    lengths = draw_lengths(spec, per, gen)
    if weak and world > 1:
        lengths = lengths.repeat(world)
    mine = lpt_shard(lengths, world)[rank] if world > 1 else torch.arange(total)
    ctx = lengths[mine]
    bps = ((ctx + spec.block_size - 1) // spec.block_size).tolist()
    need = sum(bps)
    num_blocks = spec.pool_blocks or max(1, math.ceil(spec.pool_factor * need))
    bgen = torch.Generator().manual_seed(seed * 1000003 + rank + 1)
    width = max(1, math.ceil(max(spec.len_hi, int(ctx.max()) if len(ctx) else 1) / spec.block_size))
    tables = assign_blocks(bps, num_blocks, bgen, width)
    return DecodeWorkload(spec, mine, ctx.to(torch.int32), tables, num_blocks, seed)


def fill_pool(
    num_blocks: int, spec: DecodeSpec, dtype: torch.dtype, device: torch.device, seed: int,
    layers: int = 1,
) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V pools [layers, num_blocks, Hkv, bs, D] ~ value_scale * N(0, 1)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    shape = (layers, num_blocks, spec.num_kv_heads, spec.block_size, spec.head_dim)
    k = torch.empty(shape, dtype=dtype, device=device)
    v = torch.empty(shape, dtype=dtype, device=device)
    k.normal_(0.0, spec.value_scale, generator=gen)
    v.normal_(0.0, spec.value_scale, generator=gen)
    return k, v


# --------------------------------------------------------------------------- append
@dataclass
class AppendWorkload:
    """KV append of one step: decode tokens + prefill chunks, one call per layer."""

    num_layers: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    slot_mapping: torch.Tensor  # int64 [T]
    positions: torch.Tensor  # int64 [T]
    rope_theta: float

    @property
    def num_tokens(self) -> int:
        return int(self.slot_mapping.shape[0])

    def algorithmic_bytes_per_layer(self, elem: int = 2) -> int:
        """K,V read + K,V written + int64 slot and position per token."""
        row = self.num_kv_heads * self.head_dim * elem
        return self.num_tokens * (4 * row + 16)


def append_workload(
    seed: int = 0, decode_seqs: int = 256, prefill_seqs: int = 8, prefill_len: int = 2048,
    num_layers: int = 32, num_kv_heads: int = 8, head_dim: int = 128, block_size: int = 16,
    ctx_lo: int = 512, ctx_hi: int = 4096, pool_factor: float = 1.25,
) -> AppendWorkload:
    """Slots/positions for 256 single-token decode appends + 8 prompts of 2048 tokens.

    Decode sequences have contexts ~ U[ctx_lo, ctx_hi] and append their newest
    token (position ctx-1); prefill sequences write positions 0..prefill_len-1.
    Blocks come from a seeded shuffle of a pool ``pool_factor`` x the blocks
    the sequences hold.
    """
    gen = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (decode_seqs,), generator=gen)
    bps = ((ctx + block_size - 1) // block_size).tolist() + [
        (prefill_len + block_size - 1) // block_size
    ] * prefill_seqs
    num_blocks = math.ceil(pool_factor * sum(bps))
    tables = assign_blocks(bps, num_blocks, gen)
    slots, pos = [], []
    for i in range(decode_seqs):
        p = int(ctx[i]) - 1
        slots.append(int(tables[i, p // block_size]) * block_size + p % block_size)
        pos.append(p)
    for j in range(prefill_seqs):
        row = tables[decode_seqs + j].long()
        p = torch.arange(prefill_len)
        slots.extend((row[p // block_size] * block_size + p % block_size).tolist())
        pos.extend(p.tolist())
    return AppendWorkload(num_layers, num_kv_heads, head_dim, block_size, num_blocks,
                          torch.tensor(slots, dtype=torch.int64),
                          torch.tensor(pos, dtype=torch.int64), 500000.0)


# --------------------------------------------------------------------------- prefix prefill
@dataclass
class PrefixWorkload:
    """Prefix-cached prefill with a copy-on-write fork, on one layer."""

    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    prefix_lens: torch.Tensor  # int32 [B] tokens reused from the shared prefix
    q_lens: torch.Tensor  # int32 [B] new tokens per sequence
    block_tables: torch.Tensor  # int32 [B, width]
    shared_blocks: torch.Tensor  # int32 [n_shared] the prefix's blocks
    cow_pairs: torch.Tensor  # int64 [n_cow, 2] (shared src, private dst)
    slot_mapping: torch.Tensor  # int64 [sum q_lens] slots of the new tokens
    q_starts: torch.Tensor  # int32 [B]
    shared_prefix_len: int = 1024

    @property
    def batch(self) -> int:
        return int(self.q_lens.shape[0])

    @property
    def total_q(self) -> int:
        return int(self.q_lens.sum())

    def causal_flops(self) -> int:
        """4*D*Hq per attended (query, key) pair, masked pairs not counted."""
        pairs = 0
        for c, n in zip(self.prefix_lens.tolist(), self.q_lens.tolist(), strict=True):
            pairs += n * c + n * (n + 1) // 2
        return 4 * self.head_dim * self.num_q_heads * pairs


def prefix_workload(
    seed: int = 0, batch: int = 64, shared_len: int = 1024, suffix_len: int = 512,
    n_cow: int = 8, cow_prefix_len: int = 1000, num_q_heads: int = 32, num_kv_heads: int = 8,
    head_dim: int = 128, block_size: int = 16, pool_factor: float = 1.25,
) -> PrefixWorkload:
    """64 sequences over one shared 1024-token prefix; 8 fork mid-block at 1000.

    The shared prefix occupies ``shared_len/bs`` blocks referenced by every
    table. A forking sequence reuses the prefix's first ``cow_prefix_len``
    tokens; the block holding token ``cow_prefix_len`` is shared but only
    partially valid for it, so it gets a private copy (the CoW pair) into which
    its suffix writes from offset ``cow_prefix_len % bs`` on.
    """
    gen = torch.Generator().manual_seed(seed)
    bs = block_size
    n_shared = shared_len // bs
    prefix_lens, private_blocks = [], []
    for i in range(batch):
        forks = i >= batch - n_cow
        p = cow_prefix_len if forks else shared_len
        prefix_lens.append(p)
        total = p + suffix_len
        private_blocks.append((total + bs - 1) // bs - p // bs)
    need = n_shared + sum(private_blocks)
    num_blocks = math.ceil(pool_factor * need)
    perm = torch.randperm(num_blocks, generator=gen)
    shared = perm[:n_shared].to(torch.int32)
    width = max((p + suffix_len + bs - 1) // bs for p in prefix_lens)
    tables = torch.zeros((batch, width), dtype=torch.int32)
    cursor = n_shared
    cow = []
    slots = []
    for i, p in enumerate(prefix_lens):
        full = p // bs  # blocks fully inside the reused prefix
        tables[i, :full] = shared[:full]
        n_priv = private_blocks[i]
        priv = perm[cursor : cursor + n_priv].to(torch.int32)
        cursor += n_priv
        tables[i, full : full + n_priv] = priv
        if p % bs:
            cow.append((int(shared[full]), int(priv[0])))
        pos = torch.arange(p, p + suffix_len)
        row = tables[i].long()
        slots.append(row[pos // bs] * bs + pos % bs)
    q_lens = torch.full((batch,), suffix_len, dtype=torch.int32)
    q_starts = (torch.arange(batch, dtype=torch.int32) * suffix_len).to(torch.int32)
    return PrefixWorkload(
        num_q_heads, num_kv_heads, head_dim, bs, num_blocks,
        torch.tensor(prefix_lens, dtype=torch.int32), q_lens, tables, shared,
        torch.tensor(cow, dtype=torch.int64).reshape(-1, 2), torch.cat(slots), q_starts,
        shared_len,
    )

