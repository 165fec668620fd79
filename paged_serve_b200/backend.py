"""``PagedCudaBackend``: the reference's AttentionBackend over a paged KV pool.

A drop-in for ``ContiguousAttentionBackend`` (pagedserve/attention/contiguous.py:59-228)
behind the same seam (pagedserve/attention/backend.py:138-193): identical
method signatures, the same error types for the same misuse, and outputs equal
to the contiguous path's within the attention tolerance (bit-identical KV
writes). Storage and compute differ:

* KV lives in per-layer pools ``[num_blocks, Hkv, block_size, D]``; a sequence's
  tokens are found through its block table instead of a dense slot row.
* ``begin_step`` derives, once per step and entirely on the device (no host
  sync), each sequence's cached and new token counts, the slot of every new
  token and the block tables; every layer then reuses them.
* ``forward`` = one append launch (``ps_cache_append``) + one attention
  launch (``ps_paged_decode`` for query_len 1, ``ps_paged_prefill`` otherwise),
  both hand-written sm_100a kernels behind the C ABI. There is no CPU path.

Two ways to describe a step:

* Engine-managed pages: ``StepInput.block_tables`` / ``slot_mapping`` are given
  (the fields the reference reserves for its block manager, backend.py:103-113).
* Backend-managed pages (the reference's static-batching engine, which fills
  neither field): sequence slot i owns blocks ``[i*M, (i+1)*M)`` with
  ``M = ceil(max_seq_len / block_size)``, and real tokens are stored
  contiguously in logical order with left padding dropped.

In both, per-sequence lengths come from ``padding_mask`` exactly as the
contiguous backend's mask does (contiguous.py:136-169): keys attended =
real tokens in ``[0, key_len)``; new tokens = real tokens in
``[context_len, key_len)``, which under left padding are the last ones.

A third entry, :meth:`PagedCudaBackend.begin_plan`, takes a
:class:`~paged_serve_b200.block_manager.StepPlan` from the block manager
(continuous batching: every sequence at its own length, prefix-cache hits and
copy-on-write): one pinned upload of the tables and lengths, one launch of the
copy-on-write block copies over all layers, one launch that builds the slots
and positions on the device.
"""

from __future__ import annotations

import dataclasses
import logging
import math
from array import array
from dataclasses import dataclass

import torch

from paged_serve_b200 import _lib, ops
from paged_serve_b200.block_manager import BlockManager, StepPlan
from paged_serve_b200.interface import AttentionBackend, AttentionMetadata, KVMemoryStats
from paged_serve_b200.rope import cos_sin_table

logger = logging.getLogger(__name__)

__all__ = ["PagedCudaBackend", "PagedMetadata"]


@dataclass(frozen=True)
class PagedMetadata(AttentionMetadata):
    """Per-step state shared by every layer (all tensors on the backend's device)."""

    query_len: int
    context_len: int
    key_len: int
    num_seqs: int
    block_tables: torch.Tensor  # int32 [B, W]
    slot_mapping: torch.Tensor  # int64 [B * query_len], -1 = padding
    positions: torch.Tensor  # int64 [B * query_len] logical token positions, -1 = padding
    ctx_lens: torch.Tensor  # int32 [B] keys attended by each sequence's last query
    ctx_before: torch.Tensor  # int32 [B] keys cached before this step
    q_lens: torch.Tensor  # int32 [B] real new tokens
    q_starts: torch.Tensor  # int32 [B] first real row in the flattened [B*query_len] rows
    live_tokens: torch.Tensor  # int64 [] real tokens after the step (seq_lens.sum())
    # int32 [B] longest-first launch order of a decode step (ops.decode_order), shared
    # by every layer's decode; None for prefill steps.
    seq_order: torch.Tensor | None = None
    # Mixed steps (some sequences add one token, others several), from begin_plan:
    # the one-token sequences, longest first, attend through the decode kernel
    # (int32 [n]); the prefill kernel sees prefill_q_lens, where they are 0.
    decode_list: torch.Tensor | None = None
    prefill_q_lens: torch.Tensor | None = None
    num_prefill_seqs: int = 0
    # A decode step's split-K unit list is planned once for all its layers (by
    # begin_step / begin_plan / the static loaders); forward then skips the plan.
    decode_planned: bool = False
    # Prefill steps with few query tiles over long contexts: keys per split-K
    # piece (ops.prefill_split_keys; 0 = items run whole).
    prefill_split_keys: int = 0


class PagedCudaBackend(AttentionBackend):
    """Paged KV cache with hand-written sm_100a append / decode / prefill kernels."""

    name = "paged_cuda"

    def __init__(
        self,
        model,
        *,
        device: torch.device | str,
        dtype: torch.dtype,
        cache=None,
        block_size: int | None = None,
        num_blocks: int | None = None,
        split_tokens: int = 512,
        debug_invariants: bool = False,
        split_mixed_steps: bool = True,
        overlap_mixed_steps: bool = True,
        split_prefill: bool = True,
    ) -> None:
        """
        Args:
            model: object with ``num_layers``, ``num_q_heads``, ``num_kv_heads``,
                ``head_dim`` (and optionally ``rope_theta``) — the reference's
                ``ModelConfig`` or :class:`paged_serve_b200.config.ModelConfig`.
            device, dtype: where and in what type (bf16 or fp16) KV is stored.
            cache: optional ``CacheConfig``; its ``block_size`` is the page size.
            block_size: overrides ``cache.block_size`` (default 16).
            num_blocks: pool size per layer; default = the worst case
                ``num_seq_slots * ceil(max_seq_len / block_size)``.
            split_tokens: flash-decoding partition length (0 = never split).
            debug_invariants: validate block tables / slots on the host and check
                the kernels' device error word after every call (synchronises).
            split_mixed_steps: in a block-manager step that mixes sequences adding
                one token with sequences adding several, attend the one-token
                sequences with the decode kernel (False: every sequence goes
                through the prefill kernel, as in a pure prefill step).
            overlap_mixed_steps: in such a split step, run the decode launch on a
                second stream beside the prefill launch (both after the append;
                they write disjoint output rows), so a prefill of a few query
                tiles, which occupies only a few SMs, runs inside the decode
                instead of before it. The current stream waits for both before
                forward() returns.
            split_prefill: a prefill step whose work items (two 128-row query
                tiles of one sequence and KV head) fill less than two waves of
                SMs cuts each item's key range into pieces run by different
                CTAs and merged by a second launch (a long prompt's chunk over
                its long cached prefix); mixed steps hide their prefill under the
                decode instead and never split it.
        """
        if model.num_q_heads % model.num_kv_heads != 0:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        self.model = model
        self.device = torch.device(device)
        self.dtype = dtype
        bs = block_size or (getattr(cache, "block_size", None) if cache is not None else None) or 16
        self.block_size = int(bs)
        self.requested_blocks = num_blocks
        self.split_tokens = int(split_tokens)
        self.debug_invariants = debug_invariants
        self.split_mixed_steps = split_mixed_steps
        self.overlap_mixed_steps = overlap_mixed_steps
        self._side_stream: torch.cuda.Stream | None = None
        self.split_prefill = split_prefill
        self._prefill_ws: torch.Tensor | None = None  # split-K prefill partials, grown on demand
        self._num_sms = 0
        self.scale = 1.0 / math.sqrt(model.head_dim)
        self.k_cache: torch.Tensor | None = None
        self.v_cache: torch.Tensor | None = None
        self.num_seq_slots = 0
        self.max_seq_len = 0
        self.num_blocks = 0
        self.max_blocks_per_seq = 0
        self._identity_tables: torch.Tensor | None = None
        self._workspace: torch.Tensor | None = None
        self._decode_out: torch.Tensor | None = None
        self._rope_table: torch.Tensor | None = None
        self._live_tokens: torch.Tensor | None = None
        self.device_error: torch.Tensor | None = None
        self.host_k_cache: torch.Tensor | None = None  # pinned swap pools [L, nh, Hkv, bs, D]
        self.host_v_cache: torch.Tensor | None = None
        self.swap_max_ctas = 0  # grid cap for swap launches (0 = library default)
        self._static: dict[int, dict] = {}  # buffers behind static_decode_metadata()
        self._manager: BlockManager | None = None  # set by make_block_manager()

    # ------------------------------------------------------------------ storage
    def allocate(self, num_seq_slots: int, max_seq_len: int) -> None:
        """Reserve the pools, the identity block tables and the split-K workspace."""
        if self.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"paged_cuda stores bf16 or fp16 KV, not {self.dtype}")
        self.free()
        m = self.model
        bs = self.block_size
        self.num_seq_slots = num_seq_slots
        self.max_seq_len = max_seq_len
        self.max_blocks_per_seq = math.ceil(max_seq_len / bs)
        self.num_blocks = self.requested_blocks or num_seq_slots * self.max_blocks_per_seq
        shape = (m.num_layers, self.num_blocks, m.num_kv_heads, bs, m.head_dim)
        self.k_cache = torch.zeros(shape, device=self.device, dtype=self.dtype)
        self.v_cache = torch.zeros(shape, device=self.device, dtype=self.dtype)
        if num_seq_slots * self.max_blocks_per_seq <= self.num_blocks:
            self._identity_tables = torch.arange(
                num_seq_slots * self.max_blocks_per_seq, device=self.device, dtype=torch.int32
            ).view(num_seq_slots, self.max_blocks_per_seq)
        ws = 0
        if self.device.type == "cuda":
            ws = ops.decode_workspace_bytes(num_seq_slots, m.num_q_heads, m.head_dim, bs,
                                            self.max_blocks_per_seq, self.split_tokens)
        self._workspace = torch.empty(max(ws, 256), device=self.device, dtype=torch.uint8)
        # Decode-step outputs, one buffer per layer: forward() of a query_len-1
        # step writes here and returns a view, so the decode loop allocates nothing.
        self._decode_out = torch.empty((m.num_layers, num_seq_slots, m.num_q_heads, m.head_dim),
                                       device=self.device, dtype=self.dtype)
        self.device_error = torch.zeros(1, device=self.device, dtype=torch.int32)
        self._live_tokens = torch.zeros((), device=self.device, dtype=torch.int64)
        logger.info(
            "allocated paged KV cache: %d layers x %d blocks of %d tokens = %.1f MiB",
            m.num_layers, self.num_blocks, bs,
            2 * self.k_cache.numel() * self.k_cache.element_size() / 2**20,
        )

    def allocate_swap_space(self, num_host_blocks: int) -> None:
        """Pinned host pools of ``num_host_blocks`` blocks per layer for swap-out."""
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before allocate_swap_space()")
        shape = (self.k_cache.shape[0], num_host_blocks) + tuple(self.k_cache.shape[2:])
        self.host_k_cache = torch.empty(shape, dtype=self.dtype, pin_memory=True)
        self.host_v_cache = torch.empty(shape, dtype=self.dtype, pin_memory=True)

    def free(self) -> None:
        self._static = {}
        self._manager = None
        self.host_k_cache = None
        self.host_v_cache = None
        self.k_cache = None
        self.v_cache = None
        self._identity_tables = None
        self._workspace = None
        self._prefill_ws = None
        self._decode_out = None
        self._rope_table = None
        self._live_tokens = None
        self.device_error = None
        self.num_seq_slots = 0
        self.max_seq_len = 0
        self.num_blocks = 0

    # ------------------------------------------------------------------ per step
    def begin_step(self, step) -> PagedMetadata:
        """Derive per-sequence lengths, slots and tables once per step (device only)."""
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before begin_step()")
        if step.key_len > self.max_seq_len:
            raise ValueError(
                f"sequence length {step.key_len} exceeds the cache's max_seq_len "
                f"{self.max_seq_len}; raise CacheConfig.max_seq_len"
            )
        b = step.num_seqs
        tq = step.query_len
        key_len = step.key_len
        bs = self.block_size
        dev = self.device
        mask = step.padding_mask[:, :key_len].to(dev, non_blocking=True)
        real = mask[:, step.context_len:key_len]
        q_lens = real.sum(1, dtype=torch.int32)
        ctx_lens = mask.sum(1, dtype=torch.int32)
        ctx_before = ctx_lens - q_lens
        idx = ctx_before.unsqueeze(1) + real.cumsum(1, dtype=torch.int32) - 1  # [B, Tq]
        positions = torch.where(real, idx, -1).to(torch.int64).reshape(-1)
        if step.block_tables is None:
            if self._identity_tables is None:
                raise ValueError("no block_tables given and the pool is smaller than the "
                                 "worst case; pass StepInput.block_tables/slot_mapping")
            if b > self.num_seq_slots:
                raise ValueError(f"{b} sequences exceed the {self.num_seq_slots} allocated slots")
            tables = self._identity_tables[:b]
            blk = tables.gather(1, (idx.clamp(min=0) // bs).long()).long()
            slots = torch.where(real, blk * bs + (idx % bs).long(), -1).reshape(-1)
        else:
            if step.slot_mapping is None:
                raise ValueError("block_tables given without slot_mapping")
            tables = step.block_tables.to(dev, torch.int32, non_blocking=True).contiguous()
            slots = step.slot_mapping.to(dev, torch.int64, non_blocking=True).reshape(-1)
            if slots.numel() != b * tq:
                raise ValueError(f"slot_mapping has {slots.numel()} entries, expected {b * tq}")
            if tables.shape[1] > self.max_blocks_per_seq:
                raise ValueError("block_tables wider than max_seq_len allows")
        q_starts = (torch.arange(b, device=dev, dtype=torch.int32) * tq + (tq - q_lens)).to(
            torch.int32)
        live = step.seq_lens.to(dev, non_blocking=True).sum().to(torch.int64)
        md = PagedMetadata(
            query_len=tq, context_len=step.context_len, key_len=key_len, num_seqs=b,
            block_tables=tables, slot_mapping=slots.contiguous(), positions=positions,
            ctx_lens=ctx_lens, ctx_before=ctx_before, q_lens=q_lens, q_starts=q_starts,
            live_tokens=live, seq_order=self._decode_order(ctx_lens, tq),
        )
        self._live_tokens = live
        if self._plan_decode(md):
            md = dataclasses.replace(md, decode_planned=True)
        elif tq > 1:
            keys = self._plan_prefill_split(self._prefill_items(None, b, tq), tq, b, key_len)
            if keys:
                md = dataclasses.replace(md, prefill_split_keys=keys)
        if self.debug_invariants:
            self._validate(md)
        return md

    def _decode_order(self, ctx_lens: torch.Tensor, query_len: int) -> torch.Tensor | None:
        """Longest-first order for the step's decode launches (one launch per step)."""
        if query_len != 1 or self.device.type != "cuda" or ctx_lens.numel() == 0:
            return None
        return ops.decode_order(ctx_lens)

    def _plan_decode(self, md: PagedMetadata) -> bool:
        """Plan a decode step's split-K units once for all its layers (the kernel
        plans nothing when nothing is split); True when the step's layers may run
        planned. The step's layers must be enqueued before the next step is
        planned: they share the workspace's one plan."""
        if md.query_len != 1 or self.device.type != "cuda" or md.num_seqs == 0:
            return False
        ops.decode_plan(md.ctx_lens, self._workspace, self.model.num_q_heads,
                        self.model.head_dim, self.block_size, md.block_tables.shape[1],
                        self.split_tokens, seq_order=md.seq_order)
        return True

    def _plan_prefill_split(self, num_items: int, max_q_len: int, num_seqs: int,
                            max_keys: int) -> int:
        """Keys per split-K piece for a prefill step (0: no split), with the
        workspace for it reserved here rather than in forward()."""
        if not self.split_prefill or self.device.type != "cuda" or max_q_len <= 1:
            return 0
        if not self._num_sms:
            self._num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        keys = ops.prefill_split_keys(num_items, max_keys, self._num_sms)
        if not keys:
            return 0
        m = self.model
        bs = self.block_size
        need = ops.prefill_workspace_bytes(num_seqs, max_q_len, m.num_q_heads, m.num_kv_heads,
                                           m.head_dim, bs, -(-max_keys // bs), keys)
        if self._prefill_ws is None or self._prefill_ws.numel() < need:
            self._prefill_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return keys

    def _prefill_items(self, q_lens: list[int] | None, num_seqs: int, query_len: int) -> int:
        """Work items of a prefill launch: per sequence, pairs of 128-row query tiles
        (128 / G tokens each) times the KV heads."""
        m = self.model
        per_pair = 2 * (128 // (m.num_q_heads // m.num_kv_heads))
        lens = q_lens if q_lens is not None else [query_len] * num_seqs
        return sum(-(-n // per_pair) for n in lens) * m.num_kv_heads

    def make_block_manager(self, *, enable_prefix_caching: bool = False) -> BlockManager:
        """A block manager over this backend's pool (and swap space, if allocated)."""
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before make_block_manager()")
        host = 0 if self.host_k_cache is None else self.host_k_cache.shape[1]
        self._manager = BlockManager(self.num_blocks, self.block_size,
                                     enable_prefix_caching=enable_prefix_caching,
                                     debug_invariants=self.debug_invariants,
                                     num_host_blocks=host)
        return self._manager

    def _pairs(self, pairs: list[tuple[int, int]]) -> torch.Tensor:
        return torch.tensor(pairs, dtype=torch.int64).pin_memory().to(self.device,
                                                                      non_blocking=True)

    def apply_block_moves(self, plan: StepPlan) -> None:
        """Run a plan's swap-outs, then swap-ins, then copy-on-write copies."""
        if plan.swap_out or plan.swap_in:
            if self.host_k_cache is None:
                raise RuntimeError("the plan moves blocks but no swap space is allocated")
        if plan.swap_out:
            ops.swap_blocks(self.host_k_cache, self.host_v_cache, self.k_cache, self.v_cache,
                            self._pairs(plan.swap_out), self.swap_max_ctas, self.device_error)
        if plan.swap_in:
            ops.swap_blocks(self.k_cache, self.v_cache, self.host_k_cache, self.host_v_cache,
                            self._pairs(plan.swap_in), self.swap_max_ctas, self.device_error)
        if plan.copies:
            if self.debug_invariants:
                ops.check_block_pairs(plan.copies)
            ops.copy_blocks(self.k_cache, self.v_cache, self._pairs(plan.copies),
                            self.device_error)

    def begin_plan(self, plan: StepPlan, width: int | None = None) -> PagedMetadata | None:
        """Device metadata for a block-manager step, after running its block moves.

        Query rows are laid out ``[B, plan.query_len]`` with each sequence's new
        tokens last, like :meth:`begin_step`. ``width`` fixes the block-table
        width (e.g. ``max_blocks_per_seq``, for stable shapes); by default it is
        the longest table in the plan. Returns None (after the moves) when the
        plan schedules no tokens.
        """
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before begin_plan()")
        self.apply_block_moves(plan)
        b = len(plan.seq_ids)
        tq = plan.query_len
        if b == 0 or tq == 0:
            return None
        w = max(width or max(len(t) for t in plan.tables), 1)
        if w > self.max_blocks_per_seq or any(len(t) > w for t in plan.tables):
            raise ValueError("block table wider than max_seq_len or the requested width allows")
        dev = self.device
        lens = plan.seq_lens
        # A mixed step: sequences adding one token attend through the decode
        # kernel (longest first), the others through the prefill kernel.
        dec = []
        if tq > 1 and self.split_mixed_steps:
            dec = sorted((i for i, n in enumerate(plan.q_lens) if n == 1),
                         key=lambda i: -lens[i])
        # One pinned buffer, one upload: tables | ctx_before | q_lens | ctx_lens |
        # q_starts (| prefill q_lens | decode list, for a mixed step).
        buf = array("i", bytes(4 * b * w))
        for i, t in enumerate(plan.tables):
            buf[i * w : i * w + len(t)] = t if isinstance(t, array) else array("i", t)
        buf.extend(plan.ctx_before + plan.q_lens + lens
                   + [i * tq + tq - n for i, n in enumerate(plan.q_lens)])
        if dec:
            buf.extend([0 if n == 1 else n for n in plan.q_lens] + dec)
        host = torch.frombuffer(buf, dtype=torch.int32)
        if dev.type == "cuda":
            host = host.pin_memory()
        packed = host.to(dev, non_blocking=True)
        tables = packed[: b * w].view(b, w)
        ctx_before, q_lens, ctx_lens, q_starts = packed[b * w : b * w + 4 * b].view(4, b).unbind(0)
        decode_list = prefill_q_lens = None
        if dec:
            prefill_q_lens = packed[b * w + 4 * b : b * w + 5 * b]
            decode_list = packed[b * w + 5 * b :]
        slots, positions = ops.build_slot_mapping(tables, ctx_before, q_lens, tq, self.block_size,
                                                  self.num_blocks, True, self.device_error)
        live = torch.tensor(sum(lens), dtype=torch.int64)
        md = PagedMetadata(
            query_len=tq, context_len=max(plan.ctx_before), key_len=max(lens), num_seqs=b,
            block_tables=tables, slot_mapping=slots, positions=positions,
            ctx_lens=ctx_lens, ctx_before=ctx_before, q_lens=q_lens,
            q_starts=q_starts, live_tokens=live, seq_order=self._decode_order(ctx_lens, tq),
            decode_list=decode_list, prefill_q_lens=prefill_q_lens,
            num_prefill_seqs=sum(1 for n in plan.q_lens if n > 1),
        )
        self._live_tokens = live
        if self._plan_decode(md):
            md = dataclasses.replace(md, decode_planned=True)
        elif tq > 1 and not dec:
            keys = self._plan_prefill_split(self._prefill_items(plan.q_lens, b, tq), tq, b,
                                            max(lens))
            if keys:
                md = dataclasses.replace(md, prefill_split_keys=keys)
        if self.debug_invariants:
            self._validate(md)
            self._check_device_error()
        return md

    # ------------------------------------------------------------------ CUDA graphs
    def static_decode_metadata(self, batch: int, width: int | None = None) -> PagedMetadata:
        """Decode-step metadata in persistent device buffers, refilled in place.

        Capture a per-layer loop that calls :meth:`forward` with this metadata
        once (``torch.cuda.graph``), then before every replay refill it with
        :meth:`load_decode_plan` or :meth:`load_decode`. ``forward`` neither
        allocates outside the capture's pool nor synchronises (with
        ``debug_invariants`` off), so the graph holds only the kernels. Rows
        beyond a step's sequences are inactive (no append, zero output).
        """
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before static_decode_metadata()")
        w = width or self.max_blocks_per_seq
        if w > self.max_blocks_per_seq:
            raise ValueError("width exceeds max_blocks_per_seq")
        if batch > self.num_seq_slots and self.split_tokens:
            raise ValueError(f"a static batch of {batch} exceeds the {self.num_seq_slots} "
                             "sequence slots the split-K workspace was sized for")
        dev = self.device
        ints = torch.zeros(batch * (w + 4), dtype=torch.int32, device=dev)
        longs = torch.full((2 * batch,), -1, dtype=torch.int64, device=dev)
        ctx_before, q_lens, ctx_lens, q_starts = ints[batch * w :].view(4, batch).unbind(0)
        md = PagedMetadata(
            query_len=1, context_len=0, key_len=0, num_seqs=batch,
            block_tables=ints[: batch * w].view(batch, w), slot_mapping=longs[:batch],
            positions=longs[batch:], ctx_lens=ctx_lens, ctx_before=ctx_before, q_lens=q_lens,
            q_starts=q_starts, live_tokens=torch.zeros((), dtype=torch.int64),
            seq_order=torch.arange(batch, dtype=torch.int32, device=dev),
            decode_planned=dev.type == "cuda" and batch > 0,
        )
        pin = dev.type == "cuda"
        staging = [torch.zeros(ints.numel(), dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._static[id(md)] = {"md": md, "ints": ints, "staging": staging,
                                "events": [None, None], "turn": 0}
        self._plan_decode(md)  # every row inactive until the first load
        return md

    def _fill_static(self, md: PagedMetadata, tables, ctx_before, q_lens) -> None:
        """Write tables | ctx_before | q_lens | ctx_lens | q_starts into md's buffers.

        ``tables``: a CPU int32 tensor ``[n, <= width]`` or n int32 arrays/lists;
        ``ctx_before``/``q_lens``: n ints (list or CPU tensor).
        """
        st = self._static.get(id(md))
        if st is None:
            raise ValueError("metadata was not made by static_decode_metadata()")
        b, w = md.block_tables.shape
        ctx_t = torch.as_tensor(ctx_before, dtype=torch.int32)
        q_t = torch.as_tensor(q_lens, dtype=torch.int32)
        n = ctx_t.numel()
        if n > b:
            raise ValueError(f"{n} sequences exceed the static batch of {b}")
        if q_t.numel() and (int(q_t.min()) < 0 or int(q_t.max()) > 1):
            raise ValueError("a static decode step computes at most one token per sequence")
        turn = st["turn"]
        st["turn"] ^= 1
        if st["events"][turn] is not None:
            st["events"][turn].synchronize()  # the upload that last read this buffer is done
        host = st["staging"][turn]
        host.zero_()
        tv = host[: b * w].view(b, w)
        if isinstance(tables, torch.Tensor):
            if tables.shape[0] != n or tables.shape[1] > w:
                raise ValueError("block tables do not match the sequences or the static width")
            tv[:n, : tables.shape[1]] = tables
        else:
            buf = array("i", bytes(4 * n * w))
            for i, t in enumerate(tables):
                if len(t) > w:
                    raise ValueError("block table wider than the static metadata")
                buf[i * w : i * w + len(t)] = t if isinstance(t, array) else array("i", t)
            if n:
                tv[:n] = torch.frombuffer(buf, dtype=torch.int32).view(n, w)
        tail = host[b * w :].view(4, b)
        tail[0, :n] = ctx_t
        tail[1, :n] = q_t
        tail[2, :n] = ctx_t + q_t
        tail[3] = torch.arange(1, b + 1, dtype=torch.int32) - tail[1]
        st["ints"].copy_(host, non_blocking=True)
        ev = torch.cuda.Event() if self.device.type == "cuda" else None
        if ev is not None:
            ev.record()
        st["events"][turn] = ev
        ops.build_slot_mapping(md.block_tables, md.ctx_before, md.q_lens, 1, self.block_size,
                               self.num_blocks, True, self.device_error,
                               out=(md.slot_mapping, md.positions))
        if self.device.type == "cuda":
            ops.decode_order(md.ctx_lens, out=md.seq_order)
        self._plan_decode(md)
        md.live_tokens.fill_(int((ctx_t + q_t).sum()))
        self._live_tokens = md.live_tokens

    def load_decode_plan(self, md: PagedMetadata, plan: StepPlan) -> None:
        """Refill static decode metadata from a block-manager plan (moves run first)."""
        self.apply_block_moves(plan)
        self._fill_static(md, plan.tables, plan.ctx_before, plan.q_lens)

    def load_decode(self, md: PagedMetadata, block_tables: torch.Tensor,
                    ctx_lens: torch.Tensor) -> None:
        """Refill static decode metadata for sequences whose newest token is the step's.

        ``block_tables`` int32 ``[n, <= width]`` and ``ctx_lens`` (keys after the
        step, the new token included) on the host.
        """
        ctx = torch.as_tensor(ctx_lens, dtype=torch.int32).cpu()
        self._fill_static(md, block_tables.to(torch.int32).cpu(), (ctx - 1).clamp(min=0),
                          (ctx > 0).to(torch.int32))

    def _validate(self, md: PagedMetadata) -> None:
        """Host-side checks of the index tensors (synchronises; debug only)."""
        bs = self.block_size
        tables = md.block_tables.cpu()
        ctx = md.ctx_lens.cpu()
        need = (ctx + bs - 1) // bs
        if need.numel() and int(need.max()) > tables.shape[1]:
            raise ValueError("a sequence needs more blocks than its block table holds")
        for i in range(md.num_seqs):
            row = tables[i, : int(need[i])]
            if row.numel() and (int(row.min()) < 0 or int(row.max()) >= self.num_blocks):
                raise ValueError(f"sequence {i}: block id outside [0, {self.num_blocks})")
        slots = md.slot_mapping.cpu()
        real = slots[slots >= 0]
        if (slots < -1).any() or (real >= self.num_blocks * bs).any():
            raise ValueError("slot_mapping entry outside [-1, num_blocks*block_size)")
        if real.numel() != real.unique().numel():
            raise ValueError("slot_mapping writes one slot twice")

    def _check_device_error(self) -> None:
        if self.device_error is None:
            return
        code = int(self.device_error.item())
        if code:
            self.device_error.zero_()
            raise RuntimeError(f"paged_cuda kernel reported device error bits 0x{code:x}")

    # ------------------------------------------------------------------ compute
    def forward(
        self,
        layer_idx: int,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        metadata: AttentionMetadata,
    ) -> torch.Tensor:
        """Append this step's K/V through the slots, then attend (decode or prefill;
        a decode step does both in one launch).

        A decode step (query_len 1) allocates nothing: its output is a view of a
        per-layer buffer reserved by :meth:`allocate`, valid until this layer's
        next decode step (the model consumes it at once, layers.py:192). Prefill
        steps return a new tensor.
        """
        assert isinstance(metadata, PagedMetadata)
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before forward()")
        md = metadata
        b, tq, hq, d = query.shape
        hkv = self.model.num_kv_heads
        k_pool = self.k_cache[layer_idx]
        v_pool = self.v_cache[layer_idx]
        if tq == 1:
            # One launch: each sequence's new K/V row is written by the CTA that
            # then attends over it (same pool contents as append + decode).
            buf = None
            if self._decode_out is not None and b <= self._decode_out.shape[1]:
                buf = self._decode_out[layer_idx, :b]
            out = ops.paged_decode_append(
                query.reshape(b, hq, d), key.reshape(b, hkv, d), value.reshape(b, hkv, d),
                md.slot_mapping, k_pool, v_pool, md.block_tables, md.ctx_lens,
                self.scale, self.split_tokens, out=buf, workspace=self._workspace,
                device_error=self.device_error, seq_order=md.seq_order,
                planned=md.decode_planned,
            ).view(b, 1, hq, d)
        elif md.decode_list is not None:
            # Mixed step: one append for every new token, the prefill kernel for
            # the sequences adding several (the others have q_len 0 there), and
            # the decode kernel for those adding one, each at its last row.
            ops.cache_append(k_pool, v_pool, key.reshape(b * tq, hkv, d),
                             value.reshape(b * tq, hkv, d), md.slot_mapping, self.device_error)
            flat = query.reshape(b * tq, hq, d)
            out = torch.empty_like(flat)

            def decode() -> None:
                ops.paged_decode_listed(
                    flat.view(b, tq, hq, d)[:, tq - 1], k_pool, v_pool, md.block_tables,
                    md.ctx_lens, md.decode_list, self.scale, self.split_tokens,
                    out=out.view(b, tq, hq, d)[:, tq - 1], workspace=self._workspace,
                    device_error=self.device_error)

            side = None
            if md.num_prefill_seqs and self.overlap_mixed_steps and self.device.type == "cuda":
                # The prefill keeps the current stream (it launches first and takes
                # its SMs whole); the decode fills the rest from the side stream.
                main = torch.cuda.current_stream(self.device)
                if self._side_stream is None:
                    self._side_stream = torch.cuda.Stream(self.device)
                side = self._side_stream
                side.wait_stream(main)
            if md.num_prefill_seqs:
                ops.paged_prefill(flat, k_pool, v_pool, md.block_tables, md.q_starts,
                                  md.prefill_q_lens, md.ctx_before, tq, self.scale, out=out,
                                  device_error=self.device_error)
            if side is not None:
                with torch.cuda.stream(side):
                    decode()
                # The caller's query and the returned output are used on the side
                # stream too: keep the allocator from reusing them before it is done
                # (under graph capture they live in the graph's own pool).
                if not torch.cuda.is_current_stream_capturing():
                    flat.record_stream(side)
                    out.record_stream(side)
                main.wait_stream(side)
            else:
                decode()
            out = out.view(b, tq, hq, d)
        else:
            ops.cache_append(k_pool, v_pool, key.reshape(b * tq, hkv, d),
                             value.reshape(b * tq, hkv, d), md.slot_mapping, self.device_error)
            split = md.prefill_split_keys
            out = ops.paged_prefill(
                query.reshape(b * tq, hq, d), k_pool, v_pool, md.block_tables, md.q_starts,
                md.q_lens, md.ctx_before, tq, self.scale, device_error=self.device_error,
                split_keys=split, workspace=self._prefill_ws if split else None,
                max_keys=md.key_len,
            ).view(b, tq, hq, d)
        if self.debug_invariants:
            self._check_device_error()
        return out

    def write_kv_rope(
        self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, metadata: PagedMetadata
    ) -> None:
        """Fused RoPE + append for callers that hold un-rotated K.

        Rotates K by each token's logical position (the reference's position ids
        under left padding, pagedserve/engine.py:255-273) with the same cos/sin
        RotaryEmbedding produces on this device, and writes K/V to the pool —
        the work of ``apply_rotary`` on K plus the append, in one launch.
        """
        if self.k_cache is None:
            raise RuntimeError("allocate() must be called before write_kv_rope()")
        if self._rope_table is None:
            theta = float(getattr(self.model, "rope_theta", 10000.0))
            self._rope_table = cos_sin_table(self.model.head_dim, theta, self.max_seq_len,
                                             self.dtype, self.device)
        b, tq, hkv, d = key.shape
        ops.cache_append_rope(self.k_cache[layer_idx], self.v_cache[layer_idx],
                              key.reshape(b * tq, hkv, d), value.reshape(b * tq, hkv, d),
                              metadata.slot_mapping, metadata.positions, self._rope_table,
                              self.device_error)

    # ------------------------------------------------------------------ stats
    def memory_stats(self) -> KVMemoryStats:
        """Reserved versus live KV bytes, the reference's definition
        (pagedserve/attention/backend.py:44-66, contiguous.py:211-227).

        allocated = the K and V pools this backend reserved in ``allocate()``
        (all layers), whether the backend pages sequences itself (static
        batching) or a block manager hands out the blocks; live = token slots
        that hold real K/V x per-token KV bytes (with a block manager, a prefix
        block shared through the cache is counted once). :meth:`block_usage`
        reports the blocks sequences hold.
        """
        if self.k_cache is None:
            return KVMemoryStats(allocated_bytes=0, live_bytes=0)
        per_token = self._kv_bytes_per_token()
        allocated = 2 * self.k_cache.numel() * self.k_cache.element_size()
        if self._manager is not None:
            return KVMemoryStats(allocated_bytes=allocated,
                                 live_bytes=self._manager.physical_tokens() * per_token)
        live = int(self._live_tokens.item()) if self._live_tokens is not None else 0
        return KVMemoryStats(allocated_bytes=allocated, live_bytes=live * per_token)

    def block_usage(self) -> dict[str, int]:
        """Pool blocks: total, held by sequences (block manager) and their bytes."""
        if self.k_cache is None:
            return {"num_blocks": 0, "held_blocks": 0, "held_bytes": 0}
        held = self._manager.num_used_blocks if self._manager is not None else self.num_blocks
        return {"num_blocks": self.num_blocks, "held_blocks": held,
                "held_bytes": held * self.block_size * self._kv_bytes_per_token()}

    def _kv_bytes_per_token(self) -> int:
        m = self.model
        return 2 * m.num_layers * m.num_kv_heads * m.head_dim * self.k_cache.element_size()

def native_library_loaded() -> bool:
    """True once the C-ABI library has been loaded into this process."""
    return _lib._lib is not None


def register_with_reference_seam() -> bool:
    """Register :class:`PagedCudaBackend` as a virtual subclass of the reference's
    ``pagedserve.attention.backend.AttentionBackend`` when that package is
    importable, so ``isinstance`` checks written against the reference's seam
    accept it. Returns whether the reference was found. Called once at import;
    call again after putting the reference on ``sys.path``.
    """
    import importlib.util

    try:
        if importlib.util.find_spec("pagedserve") is None:
            return False
        from pagedserve.attention.backend import AttentionBackend as ReferenceBackend
    except Exception:  # the reference is optional: any import failure means "absent"
        return False
    ReferenceBackend.register(PagedCudaBackend)
    return True


register_with_reference_seam()

