"""Block manager and prefix cache: the producers of block tables, slots and CoW copies.

The reference plans these (``memory/block_manager.py``: "free list, block tables,
refcounts, alloc/free/fork"; ``memory/prefix_cache.py``: "hash chain, LRU
evictor"; AGENTS.md) but has not written them. They are built here to the
reference's stated contract so that the paged kernels can be driven end to end:

* Physical blocks hold ``block_size`` token slots of every layer's K/V.
* A sequence owns a block table: logical block i of the sequence lives in
  physical block ``table[i]``; token t sits in slot ``table[t // bs]*bs + t % bs``.
* Blocks are refcounted. ``fork`` makes a child share all of its parent's blocks;
  writing into a block whose refcount is above one first copies it to a private
  block (copy-on-write) — the (src, dst) pair goes to ``ps_copy_blocks``.
* With prefix caching on, every *full* block is keyed by a hash chain over the
  token ids it holds and everything before it, so sequences with a common
  block-aligned prefix share those blocks. A block becomes findable only once
  a step that writes all of its K/V has been scheduled (:meth:`schedule`):
  until then its hash waits in a pending map. Steps run in the order they are
  scheduled, on one stream, so those writes precede every later reader. A
  cached block whose refcount drops to zero stays findable on an LRU list and
  is evicted only when a fresh block is needed and the free list is empty.

* Preemption (the reference's RECOMPUTE | SWAP policies): :meth:`preempt`
  frees a sequence and returns its token ids for re-admission (recompute; the
  prefix cache then finds its full blocks if they were not evicted), and
  :meth:`swap_out` / :meth:`swap_in` move a sequence's blocks to and from a
  pool of host blocks. The block moves come out with the next plan, to run
  before that step's copy-on-write copies: swap-outs first (they read HBM
  blocks that may be handed out again in the same step), then swap-ins. Host
  blocks released by a swap-in or a free are reused only after the next plan
  is built, so no plan writes a host block that the same plan still reads.

Invariants (the reference's debug list, checked by :meth:`check_invariants`):
the sum of refcounts equals the number of block references held by sequences;
``len(free) + len(in_use) + len(evictable) == num_blocks``; a sequence's table
length is ``ceil(len(sequence) / block_size)``; no sequence holds a block with
refcount zero.
"""

from __future__ import annotations

import hashlib
from array import array
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

__all__ = ["BlockManager", "NoFreeBlocksError", "StepPlan"]


class NoFreeBlocksError(RuntimeError):
    """The pool has no free or evictable block left."""


@dataclass
class _Seq:
    table: array = field(default_factory=lambda: array("i"))  # int32 block ids
    tokens: list[int] = field(default_factory=list)  # token ids (for prefix hashing)
    length: int = 0  # tokens with a reserved slot
    computed: int = 0  # leading tokens whose K/V is written (or scheduled in an issued step)
    hashes: list[bytes] = field(default_factory=list)  # chain hash of each full block
    host_table: array | None = None  # host block ids while swapped out


@dataclass
class StepPlan:
    """One step's host-side schedule: which tokens of which sequences to compute.

    Sequence ``seq_ids[i]`` computes ``q_lens[i]`` new tokens at logical
    positions ``[ctx_before[i], ctx_before[i] + q_lens[i])`` through block table
    ``tables[i]``; ``copies`` are copy-on-write ``(src, dst)`` block pairs that
    must run before the step writes K/V. ``PagedCudaBackend.begin_plan`` turns a
    plan into device tensors (slots built on the device).
    """

    seq_ids: list[int]
    tables: list[array]  # int32 block ids per sequence (copies, safe to keep)
    ctx_before: list[int]
    q_lens: list[int]
    copies: list[tuple[int, int]]
    swap_out: list[tuple[int, int]] = field(default_factory=list)  # (HBM block, host block)
    swap_in: list[tuple[int, int]] = field(default_factory=list)  # (host block, HBM block)

    @property
    def query_len(self) -> int:
        """Rows per sequence in the padded ``[B, query_len]`` step layout."""
        return max(self.q_lens, default=0)

    @property
    def seq_lens(self) -> list[int]:
        return [c + n for c, n in zip(self.ctx_before, self.q_lens, strict=True)]

    def slot(self, i: int, pos: int, block_size: int) -> int:
        """Flat slot of logical token ``pos`` of the plan's i-th sequence."""
        return self.tables[i][pos // block_size] * block_size + pos % block_size


class BlockManager:
    """Free list + refcounted block tables + optional block-aligned prefix cache."""

    def __init__(
        self,
        num_blocks: int,
        block_size: int = 16,
        *,
        enable_prefix_caching: bool = False,
        debug_invariants: bool = False,
        free_order: list[int] | None = None,
        num_host_blocks: int = 0,
    ) -> None:
        """``free_order``: the order in which never-used blocks are handed out
        (a permutation of ``range(num_blocks)``; default low ids first).
        ``num_host_blocks``: size of the host swap pool (0 = no swapping)."""
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        if free_order is not None and sorted(free_order) != list(range(num_blocks)):
            raise ValueError("free_order must be a permutation of range(num_blocks)")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_caching = enable_prefix_caching
        self.debug_invariants = debug_invariants
        self.refcount = [0] * num_blocks
        # Blocks are popped from the end of the free list.
        order = free_order if free_order is not None else range(num_blocks)
        self._free: list[int] = list(reversed(list(order)))
        self._seqs: dict[int, _Seq] = {}
        self._cached: dict[bytes, int] = {}  # chain hash -> block
        self._block_hash: dict[int, bytes] = {}  # block -> chain hash (cached blocks only)
        self._evictable: OrderedDict[int, None] = OrderedDict()  # LRU: oldest first
        self._pending: dict[int, bytes] = {}  # block -> hash, K/V not yet issued
        self.pending_copies: list[tuple[int, int]] = []
        self.num_host_blocks = num_host_blocks
        self._host_free: list[int] = list(range(num_host_blocks - 1, -1, -1))
        self._host_released: list[int] = []  # reusable once the next plan is built
        self._swap_out: list[tuple[int, int]] = []
        self._swap_in: list[tuple[int, int]] = []
        self.hits = 0
        self.misses = 0

    # ------------------------------------------------------------------ queries
    @property
    def num_free_blocks(self) -> int:
        """Blocks that can be handed out now (free + evictable cached)."""
        return len(self._free) + len(self._evictable)

    def has_seq(self, seq_id: int) -> bool:
        return seq_id in self._seqs

    def block_table(self, seq_id: int) -> list[int]:
        return list(self._seqs[seq_id].table)

    def seq_len(self, seq_id: int) -> int:
        return self._seqs[seq_id].length

    def num_computed(self, seq_id: int) -> int:
        """Leading tokens of the sequence whose K/V needs no computing this step."""
        return self._seqs[seq_id].computed

    @property
    def num_used_blocks(self) -> int:
        """Blocks held by sequences (cached blocks nobody holds are reclaimable)."""
        return self.num_blocks - self.num_free_blocks

    def physical_tokens(self) -> int:
        """Token slots holding K/V in HBM, a block shared by several sequences counted once."""
        filled: dict[int, int] = {}
        bs = self.block_size
        for s in self._seqs.values():
            if s.host_table is not None:
                continue
            for i, blk in enumerate(s.table):
                n = min(bs, s.length - i * bs)
                if n > filled.get(blk, 0):
                    filled[blk] = n
        return sum(filled.values())

    def blocks_needed(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    def can_allocate(self, num_tokens: int) -> bool:
        return self.blocks_needed(num_tokens) <= self.num_free_blocks

    # ------------------------------------------------------------------ block pool
    def _take_block(self) -> int:
        if self._free:
            blk = self._free.pop()
        elif self._evictable:
            blk, _ = self._evictable.popitem(last=False)  # least recently used
            h = self._block_hash.pop(blk)
            del self._cached[h]
        else:
            raise NoFreeBlocksError("no free KV blocks")
        self.refcount[blk] = 1
        return blk

    def _release(self, blk: int) -> None:
        self.refcount[blk] -= 1
        if self.refcount[blk] > 0:
            return
        self._pending.pop(blk, None)  # its K/V is no longer wanted
        if self.pending_copies:  # nor a copy-on-write into it that has not run yet
            self.pending_copies = [c for c in self.pending_copies if c[1] != blk]
        if blk in self._block_hash:
            self._evictable[blk] = None  # stays findable until evicted
        else:
            self._free.append(blk)

    def _acquire_cached(self, blk: int) -> None:
        if self.refcount[blk] == 0:
            self._evictable.pop(blk, None)
        self.refcount[blk] += 1

    # ------------------------------------------------------------------ hashing
    def _chain(self, prev: bytes, tokens: list[int]) -> bytes:
        h = hashlib.blake2b(prev, digest_size=16)
        h.update(array("q", tokens).tobytes())
        return h.digest()

    # ------------------------------------------------------------------ sequence ops
    def allocate(self, seq_id: int, num_tokens: int, token_ids: list[int] | None = None) -> list[int]:
        """Create a sequence holding ``num_tokens`` tokens (its prompt).

        With prefix caching and ``token_ids``, leading full blocks whose chain
        hash is cached (and published) are shared instead of allocated, and
        count as computed. A hit never covers the whole prompt: the final block
        is recomputed so the last token's attention is produced. Returns the
        block table.
        """
        if seq_id in self._seqs:
            raise ValueError(f"sequence {seq_id} already exists")
        if token_ids is not None and len(token_ids) != num_tokens:
            raise ValueError("token_ids must hold num_tokens ids")
        bs = self.block_size
        s = _Seq(tokens=list(token_ids) if token_ids is not None else [], length=num_tokens)
        need = self.blocks_needed(num_tokens)
        hits: list[int] = []  # leading cached blocks (never the last block of the prompt)
        if self.enable_prefix_caching and token_ids is not None:
            prev = b""
            for i in range(num_tokens // bs):
                prev = self._chain(prev, s.tokens[i * bs : (i + 1) * bs])
                s.hashes.append(prev)
                blk = self._cached.get(prev)
                if blk is not None and len(hits) == i and (i + 1) * bs < num_tokens:
                    hits.append(blk)
        # Check capacity before touching any state, so a failed call changes nothing
        # (in particular it evicts no cached block).
        revived = sum(1 for blk in hits if self.refcount[blk] == 0)
        if need - len(hits) > len(self._free) + len(self._evictable) - revived:
            raise NoFreeBlocksError(
                f"sequence {seq_id} needs {need - len(hits)} new blocks, "
                f"{self.num_free_blocks - revived} available")
        for blk in hits:
            self._acquire_cached(blk)
        fresh = [self._take_block() for _ in range(need - len(hits))]
        s.table = array("i", hits + fresh)
        s.computed = len(hits) * bs
        self.hits += len(hits)
        self.misses += len(s.hashes) - len(hits)
        for i in range(len(hits), len(s.hashes)):
            self._pending[s.table[i]] = s.hashes[i]
        self._seqs[seq_id] = s
        self._check()
        return list(s.table)

    def append_slots(self, seq_id: int, n: int = 1, token_ids: list[int] | None = None) -> list[int]:
        """Reserve slots for ``n`` new tokens at the end of the sequence.

        Allocates blocks as the sequence crosses block boundaries; if the block
        being written is shared (refcount > 1) it is first copied to a private
        block (copy-on-write) and the pair is queued in ``pending_copies``.
        Returns the flat slot of each new token.
        """
        s = self._resident(seq_id)
        bs = self.block_size
        slots = []
        for k in range(n):
            t = s.length
            i = t // bs
            if i == len(s.table):
                s.table.append(self._take_block())
            elif self.refcount[s.table[i]] > 1:
                src = s.table[i]
                dst = self._take_block()
                self.refcount[src] -= 1
                s.table[i] = dst
                self.pending_copies.append((src, dst))
            slots.append(s.table[i] * bs + t % bs)
            s.length += 1
            if token_ids is not None:
                s.tokens.append(token_ids[k])
            if self.enable_prefix_caching and s.length % bs == 0 and token_ids is not None:
                self._register_full_block(s, s.length // bs - 1)
        self._check()
        return slots

    def _register_full_block(self, s: _Seq, i: int) -> None:
        """Publish a block that just became full in the prefix cache (if new)."""
        prev = s.hashes[i - 1] if i > 0 else b""
        if len(s.hashes) != i:
            return  # an earlier block of this sequence was never hashed
        h = self._chain(prev, s.tokens[i * self.block_size : (i + 1) * self.block_size])
        s.hashes.append(h)
        blk = s.table[i]
        if h not in self._cached and blk not in self._block_hash:
            self._pending[blk] = h

    def _publish(self, s: _Seq) -> None:
        """Make the sequence's full blocks whose K/V is scheduled findable."""
        for i in range(min(s.computed // self.block_size, len(s.hashes))):
            blk = s.table[i]
            h = self._pending.get(blk)
            if h is None:
                continue
            del self._pending[blk]
            if h not in self._cached and blk not in self._block_hash:
                self._cached[h] = blk
                self._block_hash[blk] = h

    def _resident(self, seq_id: int) -> _Seq:
        s = self._seqs[seq_id]
        if s.host_table is not None:
            raise ValueError(f"sequence {seq_id} is swapped out")
        return s

    def is_swapped(self, seq_id: int) -> bool:
        return self._seqs[seq_id].host_table is not None

    @property
    def num_free_host_blocks(self) -> int:
        return len(self._host_free)

    def tokens(self, seq_id: int) -> list[int]:
        return list(self._seqs[seq_id].tokens)

    # ------------------------------------------------------------------ preemption
    def preempt(self, seq_id: int) -> list[int]:
        """RECOMPUTE preemption: drop the sequence, return its token ids to re-admit."""
        toks = self.tokens(seq_id)
        self.free(seq_id)
        return toks

    def swap_out(self, seq_id: int) -> list[tuple[int, int]]:
        """SWAP preemption: move the sequence's blocks to host blocks.

        Only a sequence whose tokens are all scheduled can leave (its K/V is
        then written, or will be by steps that run before the move). Raises
        :class:`NoFreeBlocksError` and changes nothing if the host pool is too
        small. Returns the queued (HBM block, host block) pairs.
        """
        s = self._resident(seq_id)
        if s.computed != s.length:
            raise ValueError("swap out a sequence only after all of its tokens are scheduled")
        if len(s.table) > len(self._host_free):
            raise NoFreeBlocksError(
                f"sequence {seq_id} needs {len(s.table)} host blocks, "
                f"{len(self._host_free)} free")
        pairs = [(blk, self._host_free.pop()) for blk in s.table]
        for blk in s.table:
            self._release(blk)
        s.host_table = array("i", [h for _, h in pairs])
        s.table = array("i")
        self._swap_out.extend(pairs)
        self._check()
        return pairs

    def swap_in(self, seq_id: int) -> list[tuple[int, int]]:
        """Bring a swapped-out sequence back into HBM blocks.

        A full block whose chain hash is still cached in HBM is shared again
        instead of copied. Raises :class:`NoFreeBlocksError` and changes nothing
        if HBM blocks run short. Returns the queued (host block, HBM block) pairs.
        """
        s = self._seqs[seq_id]
        if s.host_table is None:
            raise ValueError(f"sequence {seq_id} is not swapped out")
        n = len(s.host_table)
        cached = [self._cached.get(s.hashes[i]) if self.enable_prefix_caching and
                  i < len(s.hashes) else None for i in range(n)]
        revived = sum(1 for blk in cached if blk is not None and self.refcount[blk] == 0)
        fresh_needed = sum(1 for blk in cached if blk is None)
        if fresh_needed > len(self._free) + len(self._evictable) - revived:
            raise NoFreeBlocksError(f"sequence {seq_id} needs {fresh_needed} blocks to swap in")
        for blk in cached:
            if blk is not None:
                self._acquire_cached(blk)
        table, pairs = [], []
        for i, blk in enumerate(cached):
            if blk is None:
                blk = self._take_block()
                pairs.append((s.host_table[i], blk))
                if i < len(s.hashes):
                    self._pending[blk] = s.hashes[i]
            table.append(blk)
        self._host_released.extend(s.host_table)
        s.table = array("i", table)
        s.host_table = None
        self._swap_in.extend(pairs)
        self._check()
        return pairs

    def fork(self, parent_id: int, child_id: int) -> None:
        """The child shares every block of the parent (refcounts go up)."""
        if child_id in self._seqs:
            raise ValueError(f"sequence {child_id} already exists")
        p = self._resident(parent_id)
        if p.computed != p.length:
            raise ValueError("fork a sequence only after all of its tokens are scheduled")
        for blk in p.table:
            self.refcount[blk] += 1
        self._seqs[child_id] = _Seq(table=array("i", p.table), tokens=list(p.tokens), length=p.length,
                                    computed=p.computed, hashes=list(p.hashes))
        self._check()

    def truncate_to(self, seq_id: int, num_tokens: int) -> None:
        """Keep only the first ``num_tokens`` tokens (e.g. a shared-prefix reuse point)."""
        s = self._resident(seq_id)
        if num_tokens > s.length:
            raise ValueError("cannot grow a sequence with truncate_to")
        keep = self.blocks_needed(num_tokens)
        for blk in s.table[keep:]:
            self._release(blk)
        s.table = s.table[:keep]
        s.length = num_tokens
        s.computed = min(s.computed, num_tokens)
        s.tokens = s.tokens[:num_tokens]
        s.hashes = s.hashes[: num_tokens // self.block_size]
        self._check()

    def free(self, seq_id: int) -> None:
        """Drop the sequence; blocks whose refcount reaches zero are released."""
        s = self._seqs.pop(seq_id)
        if s.host_table is not None:
            gone = set(s.host_table)
            self._swap_out = [p for p in self._swap_out if p[1] not in gone]
            self._host_released.extend(s.host_table)
        for blk in s.table:
            self._release(blk)
        self._check()

    def take_copies(self) -> list[tuple[int, int]]:
        """The copy-on-write pairs queued since the last call (run them before writing)."""
        out, self.pending_copies = self.pending_copies, []
        return out

    # ------------------------------------------------------------------ scheduling
    def schedule(self, seq_ids: list[int]) -> StepPlan:
        """Schedule every uncomputed token of ``seq_ids`` as one step.

        A sequence's new tokens are ``[computed, length)`` — the prompt suffix
        after prefix-cache hits for a new sequence, or the tokens added by
        :meth:`append_slots` for a running one. Afterwards those tokens count as
        computed, and the full blocks they complete become findable by the
        prefix cache. The CoW copies queued since the last step come along.
        """
        if len(set(seq_ids)) != len(seq_ids):
            raise ValueError("a sequence appears twice in one step")
        seqs = [self._resident(sid) for sid in seq_ids]
        plan = StepPlan(
            seq_ids=list(seq_ids),
            tables=[array("i", s.table) for s in seqs],
            ctx_before=[s.computed for s in seqs],
            q_lens=[s.length - s.computed for s in seqs],
            copies=self.take_copies(),
            swap_out=self._swap_out,
            swap_in=self._swap_in,
        )
        self._swap_out, self._swap_in = [], []
        self._host_free.extend(self._host_released)
        self._host_released = []
        for s in seqs:
            s.computed = s.length
            if self.enable_prefix_caching:
                self._publish(s)
        self._check()
        return plan

    # ------------------------------------------------------------------ invariants
    def check_invariants(self) -> None:
        refs: dict[int, int] = {}
        host_held: list[int] = []
        for sid, s in self._seqs.items():
            if s.host_table is not None:
                if s.table or len(s.host_table) != self.blocks_needed(s.length):
                    raise AssertionError(f"seq {sid}: swapped table does not cover {s.length}")
                host_held.extend(s.host_table)
                continue
            if len(s.table) != self.blocks_needed(s.length):
                raise AssertionError(f"seq {sid}: {len(s.table)} blocks for {s.length} tokens")
            if not 0 <= s.computed <= s.length:
                raise AssertionError(f"seq {sid}: computed {s.computed} outside [0, {s.length}]")
            for blk in s.table:
                refs[blk] = refs.get(blk, 0) + 1
                if self.refcount[blk] == 0:
                    raise AssertionError(f"seq {sid} holds block {blk} with refcount 0")
        if sum(self.refcount) != sum(refs.values()):
            raise AssertionError("sum of refcounts != block references held by sequences")
        for blk, n in refs.items():
            if self.refcount[blk] != n:
                raise AssertionError(f"block {blk}: refcount {self.refcount[blk]} != {n} holders")
        in_use = sum(1 for r in self.refcount if r > 0)
        if len(self._free) + in_use + len(self._evictable) != self.num_blocks:
            raise AssertionError("free + in-use + evictable != num_blocks")
        if set(self._free) & set(self._evictable):
            raise AssertionError("a block is both free and evictable")
        host_all = host_held + self._host_free + self._host_released
        if sorted(host_all) != list(range(self.num_host_blocks)):
            raise AssertionError("host blocks: held + free + released != the host pool")

    def _check(self) -> None:
        if self.debug_invariants:
            self.check_invariants()
