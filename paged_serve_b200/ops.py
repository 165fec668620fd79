"""Tensor-level entry points over the C ABI (one function per exported kernel).

Each function validates shapes/dtypes/devices on the host, extracts raw
pointers and strides, and launches on the tensor's current CUDA stream. None
of them synchronises or allocates except where an ``out=`` buffer is omitted.
There is no fallback path: a CPU tensor or a missing library raises.

KV pool layout (per layer): ``[num_blocks, num_kv_heads, block_size, head_dim]``.
"""

from __future__ import annotations

import math

import torch

from paged_serve_b200 import _lib

__all__ = [
    "build_slot_mapping",
    "cache_append",
    "cache_append_rope",
    "copy_blocks",
    "check_block_pairs",
    "decode_plan",
    "decode_workspace_bytes",
    "paged_decode",
    "paged_decode_listed",
    "paged_prefill",
    "stream_read",
    "swap_blocks",
]

_DTYPES = {torch.bfloat16: _lib.PS_DTYPE_BF16, torch.float16: _lib.PS_DTYPE_F16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; the CUDA path runs bf16 or fp16") from None


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("paged_serve_b200 kernels need CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    assert dev is not None
    return dev


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_pool(pool: torch.Tensor, name: str) -> None:
    if pool.dim() != 4 or not pool.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [num_blocks, kv_heads, block_size, head_dim]")


def _check_rows(x: torch.Tensor, name: str, heads: int, head_dim: int) -> int:
    """x is [rows, heads, head_dim] with unit dim stride and head stride head_dim."""
    if x.dim() != 3 or x.shape[1] != heads or x.shape[2] != head_dim:
        raise ValueError(f"{name} must be [rows, {heads}, {head_dim}], got {tuple(x.shape)}")
    if x.stride(2) != 1 or x.stride(1) != head_dim:
        raise ValueError(f"{name} must have contiguous heads (strides (*, {head_dim}, 1))")
    return x.stride(0) if x.shape[0] > 1 else heads * head_dim


def _err_ptr(device_error: torch.Tensor | None) -> int | None:
    if device_error is None:
        return None
    if device_error.dtype != torch.int32 or device_error.numel() < 1:
        raise ValueError("device_error must be an int32 tensor with at least one element")
    return device_error.data_ptr()


def cache_append(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    device_error: torch.Tensor | None = None,
) -> None:
    """Scatter ``key``/``value`` ([T, Hkv, D]) into the pools at ``slot_mapping`` ([T] int64).

    The KV write of ``ContiguousAttentionBackend.forward``
    (pagedserve/attention/contiguous.py:187-189), addressed through slots.
    """
    dev = _require_cuda(k_pool, v_pool, key, value, slot_mapping, device_error)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    nb, hkv, bs, d = k_pool.shape
    if v_pool.shape != k_pool.shape or key.dtype != k_pool.dtype or value.dtype != k_pool.dtype:
        raise ValueError("k_pool/v_pool/key/value must share shape and dtype")
    ks = _check_rows(key, "key", hkv, d)
    vs = _check_rows(value, "value", hkv, d)
    t = key.shape[0]
    if value.shape[0] != t or slot_mapping.shape != (t,) or slot_mapping.dtype != torch.int64:
        raise ValueError("slot_mapping must be int64 [num_tokens] matching key/value")
    if not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be contiguous")
    lib = _lib.load()
    st = lib.ps_cache_append(
        k_pool.data_ptr(), v_pool.data_ptr(), key.data_ptr(), value.data_ptr(),
        slot_mapping.data_ptr(), t, ks, vs, hkv, d, bs, nb, _dtype_code(k_pool),
        _err_ptr(device_error), _stream(dev),
    )
    _lib.check(st, "cache_append")


def cache_append_rope(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_table: torch.Tensor,
    device_error: torch.Tensor | None = None,
) -> None:
    """``cache_append`` with split-half RoPE applied to K on the way in.

    ``cos_sin_table`` is ``[max_positions, head_dim]`` in the pool dtype: row p is
    cos(p*inv_freq) then sin(p*inv_freq) (see :func:`paged_serve_b200.rope.cos_sin_table`).
    Bit-identical to the reference's ``apply_rotary`` (pagedserve/model/layers.py:62-77).
    """
    dev = _require_cuda(k_pool, v_pool, key, value, slot_mapping, positions, cos_sin_table,
                        device_error)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    nb, hkv, bs, d = k_pool.shape
    if v_pool.shape != k_pool.shape or key.dtype != k_pool.dtype or value.dtype != k_pool.dtype:
        raise ValueError("k_pool/v_pool/key/value must share shape and dtype")
    ks = _check_rows(key, "key", hkv, d)
    vs = _check_rows(value, "value", hkv, d)
    t = key.shape[0]
    if value.shape[0] != t or slot_mapping.shape != (t,) or slot_mapping.dtype != torch.int64:
        raise ValueError("slot_mapping must be int64 [num_tokens] matching key/value")
    if positions.shape != (t,) or positions.dtype != torch.int64:
        raise ValueError("positions must be int64 [num_tokens]")
    if not (slot_mapping.is_contiguous() and positions.is_contiguous()):
        raise ValueError("slot_mapping and positions must be contiguous")
    if (cos_sin_table.dim() != 2 or cos_sin_table.shape[1] != d
            or cos_sin_table.dtype != k_pool.dtype or not cos_sin_table.is_contiguous()):
        raise ValueError(f"cos_sin_table must be contiguous [positions, {d}] of the pool dtype")
    lib = _lib.load()
    st = lib.ps_cache_append_rope(
        k_pool.data_ptr(), v_pool.data_ptr(), key.data_ptr(), value.data_ptr(),
        slot_mapping.data_ptr(), positions.data_ptr(), t, ks, vs, hkv, d, bs, nb,
        cos_sin_table.data_ptr(), cos_sin_table.shape[0], d, _dtype_code(k_pool),
        _err_ptr(device_error), _stream(dev),
    )
    _lib.check(st, "cache_append_rope")


def check_block_pairs(pairs) -> None:
    """Raise ValueError unless a copy list is defined for one concurrent launch.

    ``pairs``: (src, dst) rows as a list or an [N, 2] tensor. Every destination
    must be distinct and no destination may be another pair's source; a chain
    such as (a, b), (b, c) has to be split into two calls in order.
    """
    rows = pairs.tolist() if isinstance(pairs, torch.Tensor) else [tuple(p) for p in pairs]
    dsts = [int(d) for _, d in rows]
    seen: set[int] = set()
    for d in dsts:
        if d in seen:
            raise ValueError(f"copy_blocks: destination block {d} appears twice")
        seen.add(d)
    count: dict[int, int] = {}
    for s, _ in rows:
        count[int(s)] = count.get(int(s), 0) + 1
    for s, d in rows:
        if count.get(int(d), 0) - (1 if int(s) == int(d) else 0) > 0:
            raise ValueError(f"copy_blocks: destination block {d} is another pair's source")


def copy_blocks(
    k_pools: torch.Tensor,
    v_pools: torch.Tensor,
    block_pairs: torch.Tensor,
    device_error: torch.Tensor | None = None,
    check: bool = False,
) -> None:
    """``pool[dst] = pool[src]`` for every (src, dst) row of ``block_pairs`` ([N, 2] int64).

    Pools are one layer ``[num_blocks, Hkv, bs, D]`` or all layers
    ``[L, num_blocks, Hkv, bs, D]`` (copied in one launch). All pairs run at
    once, so every destination must be distinct and none may be another
    pair's source (:func:`check_block_pairs`). ``check=True`` verifies that on
    the host first (reads the pairs back: a synchronising debug aid); the
    kernel itself flags violations in lists of up to 4096 pairs with
    ``PS_DEVERR_BLOCK_PAIRS`` in ``device_error``.
    """
    dev = _require_cuda(k_pools, v_pools, block_pairs, device_error)
    if check:
        check_block_pairs(block_pairs.cpu())
    if k_pools.shape != v_pools.shape or k_pools.dtype != v_pools.dtype:
        raise ValueError("k_pools and v_pools must match")
    if k_pools.dim() == 4:
        layers, layer_stride = 1, 0
        nb = k_pools.shape[0]
    elif k_pools.dim() == 5:
        layers = k_pools.shape[0]
        nb = k_pools.shape[1]
        layer_stride = k_pools.stride(0) * k_pools.element_size()
    else:
        raise ValueError("pools must be [blocks, Hkv, bs, D] or [L, blocks, Hkv, bs, D]")
    if not (k_pools.is_contiguous() and v_pools.is_contiguous()):
        raise ValueError("pools must be contiguous")
    if block_pairs.dtype != torch.int64 or block_pairs.dim() != 2 or block_pairs.shape[1] != 2:
        raise ValueError("block_pairs must be int64 [num_pairs, 2]")
    if not block_pairs.is_contiguous():
        raise ValueError("block_pairs must be contiguous")
    block_bytes = math.prod(k_pools.shape[-3:]) * k_pools.element_size()
    lib = _lib.load()
    st = lib.ps_copy_blocks(
        k_pools.data_ptr(), v_pools.data_ptr(), block_pairs.data_ptr(), block_pairs.shape[0],
        layers, layer_stride, block_bytes, nb, _err_ptr(device_error), _stream(dev),
    )
    _lib.check(st, "copy_blocks")


def _pool_geometry(pool: torch.Tensor) -> tuple[int, int, int]:
    """(layers, blocks, layer stride in bytes) of a [blocks, ...] or [L, blocks, ...] pool."""
    if pool.dim() == 4:
        return 1, pool.shape[0], 0
    if pool.dim() == 5:
        return pool.shape[0], pool.shape[1], pool.stride(0) * pool.element_size()
    raise ValueError("pools must be [blocks, Hkv, bs, D] or [L, blocks, Hkv, bs, D]")


def swap_blocks(
    dst_k: torch.Tensor,
    dst_v: torch.Tensor,
    src_k: torch.Tensor,
    src_v: torch.Tensor,
    block_pairs: torch.Tensor,
    max_ctas: int = 0,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """``dst[d] = src[s]`` for every (s, d) row of ``block_pairs``, K and V, all layers.

    One side is normally the device pool and the other a pinned host pool of the
    same per-block shape (swap-out: src on the device; swap-in: dst on the
    device). CPU tensors must be pinned; ``block_pairs`` (int64 ``[N, 2]``) may be
    on the device or pinned. Runs on ``stream`` (default: the current stream of
    the CUDA side) and returns without waiting.
    """
    cuda = [t for t in (dst_k, dst_v, src_k, src_v, block_pairs, device_error)
            if t is not None and t.is_cuda]
    if not cuda:
        raise ValueError("swap_blocks needs at least one CUDA pool (no CPU path)")
    dev = _require_cuda(*cuda)
    for name, t in (("dst_k", dst_k), ("dst_v", dst_v), ("src_k", src_k), ("src_v", src_v),
                    ("block_pairs", block_pairs)):
        if not t.is_cuda and not t.is_pinned():
            raise ValueError(f"{name} is pageable host memory; allocate it with pin_memory=True")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if dst_k.shape != dst_v.shape or src_k.shape != src_v.shape:
        raise ValueError("K and V pools must have the same shape on each side")
    if len({dst_k.dtype, dst_v.dtype, src_k.dtype, src_v.dtype}) != 1:
        raise ValueError("all four pools must share one dtype")
    dl, dn, dstride = _pool_geometry(dst_k)
    sl, sn, sstride = _pool_geometry(src_k)
    if dl != sl or dst_k.shape[-3:] != src_k.shape[-3:]:
        raise ValueError("source and destination pools differ in layers or block shape")
    if block_pairs.dtype != torch.int64 or block_pairs.dim() != 2 or block_pairs.shape[1] != 2:
        raise ValueError("block_pairs must be int64 [num_pairs, 2]")
    block_bytes = math.prod(dst_k.shape[-3:]) * dst_k.element_size()
    s = (stream or torch.cuda.current_stream(dev)).cuda_stream
    st = _lib.load().ps_swap_blocks(
        dst_k.data_ptr(), dst_v.data_ptr(), dn, dstride, src_k.data_ptr(), src_v.data_ptr(), sn,
        sstride, block_pairs.data_ptr(), block_pairs.shape[0], dl, block_bytes, int(max_ctas),
        _err_ptr(device_error), s,
    )
    _lib.check(st, "swap_blocks")


def build_slot_mapping(
    block_tables: torch.Tensor,
    ctx_before: torch.Tensor,
    q_lens: torch.Tensor,
    query_len: int,
    block_size: int,
    num_blocks: int,
    positions: bool = True,
    device_error: torch.Tensor | None = None,
    out: tuple[torch.Tensor, torch.Tensor | None] | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Slots (and positions) of a left-padded ``[B, query_len]`` step, on the device.

    Sequence b's ``q_lens[b]`` new tokens are its last rows and continue from
    ``ctx_before[b]`` cached tokens; padding rows get -1. ``out`` = existing
    int64 ``(slots, positions or None)`` buffers of ``B*query_len`` to fill.
    """
    dev = _require_cuda(block_tables, ctx_before, q_lens, device_error)
    b = ctx_before.shape[0]
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be int32 [num_seqs, max_blocks]")
    if block_tables.stride(1) != 1:
        raise ValueError("block_tables rows must be contiguous")
    for name, t in (("ctx_before", ctx_before), ("q_lens", q_lens)):
        if t.dtype != torch.int32 or t.shape != (b,) or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous int32 [num_seqs]")
    if out is not None:
        slots, pos = out
        for t in (slots, pos):
            if t is not None and (t.dtype != torch.int64 or t.numel() != b * query_len or
                                  not t.is_contiguous() or t.device != dev):
                raise ValueError("out buffers must be contiguous int64 [B*query_len] on the device")
    else:
        slots = torch.empty(b * query_len, dtype=torch.int64, device=dev)
        pos = torch.empty_like(slots) if positions else None
    st = _lib.load().ps_build_slot_mapping(
        slots.data_ptr(), _ptr(pos), block_tables.data_ptr(),
        block_tables.stride(0) if b > 1 else block_tables.shape[1], ctx_before.data_ptr(),
        q_lens.data_ptr(), b, int(query_len), int(block_size), block_tables.shape[1],
        int(num_blocks), _err_ptr(device_error), _stream(dev),
    )
    _lib.check(st, "build_slot_mapping")
    return slots, pos


def decode_workspace_bytes(
    num_seqs: int, num_q_heads: int, head_dim: int, block_size: int, max_blocks_per_seq: int,
    split_tokens: int,
) -> int:
    """Bytes of split-K workspace ``paged_decode`` needs (0 if nothing is split)."""
    return int(_lib.load().ps_paged_decode_workspace_bytes(
        num_seqs, num_q_heads, head_dim, block_size, max_blocks_per_seq, split_tokens))


def selftest_wait_timeout(device_error: torch.Tensor) -> None:
    """Run the shared bounded-wait failure path once: a wait on an mbarrier that
    nothing arrives at gives up after the kernels' poll bound and ORs
    ``PS_DEVERR_TIMEOUT`` into ``device_error`` (no fault, no hang)."""
    dev = _require_cuda(device_error)
    st = _lib.load().ps_selftest_wait_timeout(_err_ptr(device_error), _stream(dev))
    _lib.check(st, "selftest_wait_timeout")


def decode_order(ctx_lens: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Longest-first launch order of a decode step (int32 [B], a permutation of
    ``range(B)``), for ``paged_decode(..., seq_order=...)``; one per step serves
    every layer."""
    dev = _require_cuda(ctx_lens, out)
    if ctx_lens.dtype != torch.int32 or ctx_lens.dim() != 1 or not ctx_lens.is_contiguous():
        raise ValueError("ctx_lens must be contiguous int32 [num_seqs]")
    b = ctx_lens.shape[0]
    if out is None:
        out = torch.empty(b, dtype=torch.int32, device=dev)
    if out.dtype != torch.int32 or out.shape != (b,) or not out.is_contiguous():
        raise ValueError("out must be contiguous int32 [num_seqs]")
    st = _lib.load().ps_paged_decode_order(ctx_lens.data_ptr(), b, out.data_ptr(), _stream(dev))
    _lib.check(st, "decode_order")
    return out


class _DecodeArgs:
    """Validated arguments shared by :func:`paged_decode` and :func:`paged_decode_append`."""

    def __init__(self, query, k_pool, v_pool, block_tables, ctx_lens, out, workspace,
                 device_error, seq_order, *extra):
        self.dev = _require_cuda(query, k_pool, v_pool, block_tables, ctx_lens, out, workspace,
                                 device_error, seq_order, *extra)
        _check_pool(k_pool, "k_pool")
        _check_pool(v_pool, "v_pool")
        self.nb, self.hkv, self.bs, self.d = k_pool.shape
        d = self.d
        if v_pool.shape != k_pool.shape or query.dtype != k_pool.dtype:
            raise ValueError("k_pool/v_pool/query must share shape and dtype")
        if query.dim() != 3:
            raise ValueError("query must be [num_seqs, num_q_heads, head_dim]")
        b, hq, _ = query.shape
        self.b, self.hq = b, hq
        self.qs = _check_rows(query, "query", hq, d)
        if out is None:
            out = torch.empty((b, hq, d), dtype=query.dtype, device=self.dev)
        if out.shape != (b, hq, d) or out.dtype != query.dtype:
            raise ValueError("out must be [num_seqs, num_q_heads, head_dim] of the query dtype")
        self.out = out
        self.os = _check_rows(out, "out", hq, d)
        if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or \
                block_tables.shape[0] != b:
            raise ValueError("block_tables must be int32 [num_seqs, max_blocks]")
        if block_tables.stride(1) != 1:
            raise ValueError("block_tables rows must be contiguous")
        if ctx_lens.dtype != torch.int32 or ctx_lens.shape != (b,) or not ctx_lens.is_contiguous():
            raise ValueError("ctx_lens must be contiguous int32 [num_seqs]")
        if seq_order is not None and (seq_order.dtype != torch.int32 or seq_order.shape != (b,)
                                      or not seq_order.is_contiguous()):
            raise ValueError("seq_order must be contiguous int32 [num_seqs]")
        self.max_blocks = block_tables.shape[1]
        self.bt_stride = block_tables.stride(0) if b > 1 else self.max_blocks
        self.ws_ptr, self.ws_bytes = None, 0
        if workspace is not None:
            self.ws_ptr = workspace.data_ptr()
            self.ws_bytes = workspace.numel() * workspace.element_size()
        self.order_ptr = seq_order.data_ptr() if seq_order is not None else None


def paged_decode(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    scale: float,
    split_tokens: int = 0,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    seq_order: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode attention: ``query`` [B, Hq, D] over keys ``[0, ctx_lens[b])`` of each sequence.

    ``block_tables`` is int32 [B, max_blocks] and ``ctx_lens`` int32 [B]. Returns
    ``out`` [B, Hq, D]. With ``split_tokens`` > 0, sequences longer than one
    partition are split (flash-decoding) and ``workspace`` (uint8, at least
    :func:`decode_workspace_bytes`, 256-byte aligned) receives the partials.
    ``seq_order`` (int32 [B], from :func:`decode_order`) starts the longest
    sequences first; the result does not depend on it.
    """
    a = _DecodeArgs(query, k_pool, v_pool, block_tables, ctx_lens, out, workspace, device_error,
                    seq_order)
    st = _lib.load().ps_paged_decode_ordered(
        a.out.data_ptr(), a.os, query.data_ptr(), a.qs, k_pool.data_ptr(), v_pool.data_ptr(),
        a.nb, block_tables.data_ptr(), a.bt_stride, ctx_lens.data_ptr(), a.b, a.hq, a.hkv, a.d,
        a.bs, a.max_blocks, float(scale), int(split_tokens), a.ws_ptr, a.ws_bytes,
        _dtype_code(query), a.order_ptr, _err_ptr(device_error), _stream(a.dev),
    )
    _lib.check(st, "paged_decode")
    return a.out


def paged_decode_listed(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    seq_list: torch.Tensor,
    scale: float,
    split_tokens: int = 0,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
) -> torch.Tensor:
    """:func:`paged_decode` for the sequences in ``seq_list`` (int32 [n], indices
    into the batch, taken in that order) only; other rows of ``out`` are left
    as they are. ``query``/``out`` are [B, Hq, D] views whose rows may be strided
    (e.g. each sequence's last row of a [B, query_len, Hq, D] step)."""
    a = _DecodeArgs(query, k_pool, v_pool, block_tables, ctx_lens, out, workspace, device_error,
                    None, seq_list)
    if seq_list.dtype != torch.int32 or seq_list.dim() != 1 or not seq_list.is_contiguous():
        raise ValueError("seq_list must be contiguous int32 [n]")
    n = seq_list.shape[0]
    st = _lib.load().ps_paged_decode_listed(
        a.out.data_ptr(), a.os, query.data_ptr(), a.qs, k_pool.data_ptr(), v_pool.data_ptr(),
        a.nb, block_tables.data_ptr(), a.bt_stride, ctx_lens.data_ptr(), a.b,
        seq_list.data_ptr() if n else None, n, a.hq, a.hkv, a.d, a.bs, a.max_blocks, float(scale),
        int(split_tokens), a.ws_ptr, a.ws_bytes, _dtype_code(query), _err_ptr(device_error),
        _stream(a.dev),
    )
    _lib.check(st, "paged_decode_listed")
    return a.out


def decode_plan(
    ctx_lens: torch.Tensor,
    workspace: torch.Tensor,
    num_q_heads: int,
    head_dim: int,
    block_size: int,
    max_blocks: int,
    split_tokens: int,
    seq_order: torch.Tensor | None = None,
) -> None:
    """Plan a split-K decode step once for all its layers (``ps_paged_decode_plan``):
    the (sequence, partition) units of ``ctx_lens`` in ``seq_order`` go into
    ``workspace``; each layer then calls :func:`paged_decode_append` with
    ``planned=True``. A no-op when ``split_tokens`` splits nothing."""
    dev = _require_cuda(ctx_lens, workspace, seq_order)
    if ctx_lens.dtype != torch.int32 or ctx_lens.dim() != 1 or not ctx_lens.is_contiguous():
        raise ValueError("ctx_lens must be contiguous int32 [num_seqs]")
    b = ctx_lens.shape[0]
    if seq_order is not None and (seq_order.dtype != torch.int32 or seq_order.shape != (b,)
                                  or not seq_order.is_contiguous()):
        raise ValueError("seq_order must be contiguous int32 [num_seqs]")
    st = _lib.load().ps_paged_decode_plan(
        ctx_lens.data_ptr(), b, seq_order.data_ptr() if seq_order is not None else None,
        num_q_heads, head_dim, block_size, max_blocks, int(split_tokens), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream(dev),
    )
    _lib.check(st, "decode_plan")


def paged_decode_append(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    scale: float,
    split_tokens: int = 0,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    seq_order: torch.Tensor | None = None,
    planned: bool = False,
) -> torch.Tensor:
    """One decode step in one launch: ``cache_append`` of the step's new token
    (``key``/``value`` [B, Hkv, D], ``slot_mapping`` int64 [B], -1 = none) followed by
    :func:`paged_decode`, with the same pool contents and output. Each slot must be
    the position ``ctx_lens[b] - 1``. ``planned``: the split-K unit list for this
    step is already in ``workspace`` (:func:`decode_plan`); no plan kernel runs."""
    a = _DecodeArgs(query, k_pool, v_pool, block_tables, ctx_lens, out, workspace, device_error,
                    seq_order, key, value, slot_mapping)
    for t, name in ((key, "key"), (value, "value")):
        if t.dtype != k_pool.dtype or t.dim() != 3 or t.shape[0] != a.b:
            raise ValueError(f"{name} must be [num_seqs, num_kv_heads, head_dim] of the pool dtype")
    ks = _check_rows(key, "key", a.hkv, a.d)
    vs = _check_rows(value, "value", a.hkv, a.d)
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (a.b,) or \
            not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be contiguous int64 [num_seqs]")
    lib = _lib.load()
    fn = lib.ps_paged_decode_append_planned if planned else lib.ps_paged_decode_append
    st = fn(
        a.out.data_ptr(), a.os, query.data_ptr(), a.qs, key.data_ptr(), ks, value.data_ptr(), vs,
        slot_mapping.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), a.nb,
        block_tables.data_ptr(), a.bt_stride, ctx_lens.data_ptr(), a.b, a.hq, a.hkv, a.d, a.bs,
        a.max_blocks, float(scale), int(split_tokens), a.ws_ptr, a.ws_bytes, _dtype_code(query),
        a.order_ptr, _err_ptr(device_error), _stream(a.dev),
    )
    _lib.check(st, "paged_decode_append")
    return a.out


def prefill_workspace_bytes(
    num_seqs: int, max_q_len: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
    block_size: int, max_blocks_per_seq: int, split_keys: int,
) -> int:
    """Bytes of workspace ``paged_prefill(..., split_keys=...)`` needs (0 if nothing is split)."""
    return int(_lib.load().ps_paged_prefill_workspace_bytes(
        num_seqs, max_q_len, num_q_heads, num_kv_heads, head_dim, block_size,
        max_blocks_per_seq, split_keys))


def prefill_split_keys(num_items: int, max_keys: int, num_sms: int, min_piece_keys: int = 512,
                       max_pieces: int = 16) -> int:
    """Keys per split-K piece for a prefill of ``num_items`` work items (query-tile
    pairs x KV heads, each two tiles of 128 query rows) over at most ``max_keys``
    keys each; 0 runs every item whole.

    The prefill kernel runs one persistent CTA per SM, so fewer items than two
    waves of ``num_sms`` leave SMs idle, or a last wave half full, while each item
    walks its whole context. Cutting every item into ``pieces`` key ranges of at
    least ``min_piece_keys`` keys makes ``num_items * pieces`` units: this picks
    the fewest pieces whose units fill whole waves to 90% or more (else the best
    fill found), and no split when one piece is best.
    """
    if num_items <= 0 or num_items >= 2 * num_sms or num_sms <= 0:
        return 0
    tiles = -(-max_keys // 128)
    limit = min(max_pieces, tiles * 128 // max(min_piece_keys, 128))
    best, best_fill = 1, 0.0
    for pieces in range(1, limit + 1):
        units = num_items * pieces
        fill = units / (-(-units // num_sms) * num_sms)
        if fill > best_fill + 1e-9:
            best, best_fill = pieces, fill
        if fill >= 0.9:
            best = pieces
            break
    if best == 1:
        return 0
    return -(-tiles // best) * 128


def paged_prefill(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    q_starts: torch.Tensor,
    q_lens: torch.Tensor,
    ctx_lens: torch.Tensor,
    max_q_len: int,
    scale: float,
    out: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    split_keys: int = 0,
    workspace: torch.Tensor | None = None,
    max_keys: int | None = None,
) -> torch.Tensor:
    """Causal paged prefill over cached prefix + new tokens.

    ``query``/``out`` are [rows, Hq, D]; sequence b owns rows
    ``[q_starts[b], q_starts[b] + q_lens[b])`` and its query i attends keys
    ``[0, ctx_lens[b] + i]`` read through ``block_tables``. The new tokens' K/V
    must already be in the pools. Rows owned by no sequence are left untouched.

    ``split_keys`` > 0 cuts each work item's key range into pieces of that many
    keys (a multiple of 128) run by different CTAs and merged by a second launch
    (ps_paged_prefill_split), for prefills with few query tiles over long
    contexts. ``max_keys`` (context + new tokens of the longest sequence) bounds
    the pieces per item and so the workspace; by default the table width does.
    ``workspace`` (uint8, ``prefill_workspace_bytes`` of the same sizes) is
    allocated here when not given.
    """
    dev = _require_cuda(query, k_pool, v_pool, block_tables, q_starts, q_lens, ctx_lens, out,
                        device_error)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    nb, hkv, bs, d = k_pool.shape
    if v_pool.shape != k_pool.shape or query.dtype != k_pool.dtype:
        raise ValueError("k_pool/v_pool/query must share shape and dtype")
    if query.dim() != 3:
        raise ValueError("query must be [rows, num_q_heads, head_dim]")
    rows, hq, _ = query.shape
    qs = _check_rows(query, "query", hq, d)
    if out is None:
        out = torch.zeros((rows, hq, d), dtype=query.dtype, device=dev)
    if out.shape != (rows, hq, d) or out.dtype != query.dtype:
        raise ValueError("out must match query")
    os_ = _check_rows(out, "out", hq, d)
    b = q_starts.shape[0]
    for name, t in (("q_starts", q_starts), ("q_lens", q_lens), ("ctx_lens", ctx_lens)):
        if t.dtype != torch.int32 or t.shape != (b,) or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous int32 [num_seqs]")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be int32 [num_seqs, max_blocks]")
    if block_tables.stride(1) != 1:
        raise ValueError("block_tables rows must be contiguous")
    width = block_tables.shape[1]
    max_blocks = width
    if max_keys is not None:
        max_blocks = max(1, min(width, -(-int(max_keys) // bs)))
    bt_stride = block_tables.stride(0) if b > 1 else width
    lib = _lib.load()
    if split_keys:
        need = prefill_workspace_bytes(b, int(max_q_len), hq, hkv, d, bs, max_blocks,
                                       int(split_keys))
        if workspace is None:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        _require_cuda(workspace)
        if workspace.device != dev or not workspace.is_contiguous():
            raise ValueError("workspace must be a contiguous buffer on the query's device")
        st = lib.ps_paged_prefill_split(
            out.data_ptr(), os_, query.data_ptr(), qs, rows, k_pool.data_ptr(),
            v_pool.data_ptr(), nb, block_tables.data_ptr(), bt_stride, q_starts.data_ptr(),
            q_lens.data_ptr(), ctx_lens.data_ptr(), b, int(max_q_len), hq, hkv, d, bs, max_blocks,
            float(scale), int(split_keys), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _dtype_code(query),
            _err_ptr(device_error), _stream(dev),
        )
        _lib.check(st, "paged_prefill_split")
        return out
    st = lib.ps_paged_prefill(
        out.data_ptr(), os_, query.data_ptr(), qs, rows, k_pool.data_ptr(), v_pool.data_ptr(), nb,
        block_tables.data_ptr(), bt_stride, q_starts.data_ptr(), q_lens.data_ptr(),
        ctx_lens.data_ptr(), b, int(max_q_len), hq, hkv, d, bs, max_blocks, float(scale),
        _dtype_code(query), _err_ptr(device_error), _stream(dev),
    )
    _lib.check(st, "paged_prefill")
    return out


def stream_read(buf: torch.Tensor, checksum: torch.Tensor, method: int = _lib.PS_STREAM_BULK,
                device_error: torch.Tensor | None = None) -> None:
    """Read ``buf`` once (diagnostic HBM read stream) and XOR its 32-bit words into
    ``checksum`` (int32 [1] on the same device, zeroed by the caller).

    ``method``: ``PS_STREAM_BULK`` (bulk asynchronous copies into shared memory)
    or ``PS_STREAM_LOADS`` (16-byte loads from every thread).
    """
    dev = _require_cuda(buf, checksum, device_error)
    if not buf.is_contiguous() or checksum.dtype != torch.int32 or checksum.numel() < 1:
        raise ValueError("buf must be contiguous; checksum int32 [1]")
    nbytes = buf.numel() * buf.element_size()
    lib = _lib.load()
    st = lib.ps_stream_read(buf.data_ptr(), nbytes, checksum.data_ptr(), method,
                            _err_ptr(device_error), _stream(dev))
    _lib.check(st, "stream_read")
