"""Oracle functions (test infrastructure; see the package docstring).

Citations are to the reference project (Vivek-Chaudhari30/Paged_Serve) as
``pagedserve/<file>:<line>``. The attention math is the reference's: an
additive padding+causal bias built with ``finfo(dtype).min`` and
``torch.nn.functional.scaled_dot_product_attention`` (torch 2.11.0) over
K/V expanded per query head with ``repeat_interleave``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = [
    "contiguous_attention",
    "gather_kv",
    "oracle_append",
    "oracle_copy_blocks",
    "oracle_decode",
    "oracle_prefill",
    "rope_cos_sin",
    "rotate_half",
]


# --------------------------------------------------------------------------- attention
def contiguous_attention(
    query: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    padding_mask: torch.Tensor,
    context_len: int,
) -> torch.Tensor:
    """Attention of ``query`` over a dense, left-padded KV prefix.

    Follows ContiguousAttentionBackend: the bias of ``_build_attn_bias``
    (pagedserve/attention/contiguous.py:136-169 — keep = padding_mask[:, :key_len],
    query position = context_len + i, causal key_pos <= query_pos, disallowed
    entries = finfo(dtype).min), then the read/expand/SDPA of ``forward``
    (:191-209).

    Args:
        query: [B, Tq, Hq, D] (RoPE applied).
        keys, values: [B, key_len, Hkv, D], key_len = context_len + Tq.
        padding_mask: [B, >= key_len] bool, True on real tokens.
        context_len: tokens cached before this step (one value for the batch).

    Returns:
        [B, Tq, Hq, D] in the query dtype.
    """
    b, tq, hq, _ = query.shape
    key_len = keys.shape[1]
    assert key_len == context_len + tq, "keys must cover exactly context_len + query_len"
    dtype = query.dtype
    dev = query.device
    keep = padding_mask[:, :key_len].reshape(b, 1, 1, key_len)
    q_pos = torch.arange(context_len, context_len + tq, device=dev).reshape(1, 1, tq, 1)
    k_pos = torch.arange(key_len, device=dev).reshape(1, 1, 1, key_len)
    allowed = keep & (k_pos <= q_pos)
    bias = torch.zeros((b, 1, tq, key_len), dtype=dtype, device=dev)
    bias.masked_fill_(~allowed, torch.finfo(dtype).min)

    q = query.transpose(1, 2)
    k = keys.transpose(1, 2)
    v = values.transpose(1, 2)
    group = hq // keys.shape[2]
    if group > 1:
        k = k.repeat_interleave(group, dim=1)
        v = v.repeat_interleave(group, dim=1)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=bias).transpose(1, 2)


def gather_kv(pool: torch.Tensor, block_table: torch.Tensor, n_tokens: int) -> torch.Tensor:
    """Materialise tokens [0, n_tokens) of one sequence from a paged pool.

    ``pool`` is [num_blocks, Hkv, block_size, D]; returns [n_tokens, Hkv, D].
    This is the "gather" step the reference plans as its correctness oracle for
    a CUDA kernel (pagedserve/attention/backend.py:10-12).
    """
    bs = pool.shape[2]
    nblk = (n_tokens + bs - 1) // bs
    ids = block_table[:nblk].long()
    tiles = pool[ids]  # [nblk, Hkv, bs, D]
    return tiles.permute(0, 2, 1, 3).reshape(nblk * bs, pool.shape[1], pool.shape[3])[:n_tokens]


def oracle_decode(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    compute_dtype: torch.dtype = torch.float32,
    device: torch.device | str = "cpu",
) -> torch.Tensor:
    """Decode attention through the contiguous path.

    Each sequence's ``ctx_lens[b]`` keys (the newest one included) are gathered
    through its block table and left-padded into one dense buffer, exactly how
    the reference's static-batching engine lays out a decode step
    (pagedserve/engine.py:210-228: query at the shared last index, padding
    masked); then :func:`contiguous_attention` with query_len 1.

    Args:
        query: [B, Hq, D]. Pools: [num_blocks, Hkv, bs, D].
        compute_dtype: dtype the oracle computes in (inputs are upcast).
        device: where the same steps run: the CPU by default; a GPU device
            lets a test check a whole full-size batch in fp32 in seconds.

    Returns:
        [B, Hq, D] in ``compute_dtype`` on ``device``; rows with ctx 0 are zeros.
    """
    query = query.detach().to(device).to(compute_dtype)
    k_pool = k_pool.detach().to(device)
    v_pool = v_pool.detach().to(device)
    block_tables = block_tables.detach().to(device)
    lens = [int(x) for x in ctx_lens.detach().cpu().tolist()]
    b, hq, d = query.shape
    hkv = k_pool.shape[1]
    out = torch.zeros((b, hq, d), dtype=compute_dtype, device=device)
    live = [i for i in range(b) if lens[i] > 0]
    if not live:
        return out
    max_len = max(lens[i] for i in live)
    keys = torch.zeros((len(live), max_len, hkv, d), dtype=compute_dtype, device=device)
    values = torch.zeros_like(keys)
    mask = torch.zeros((len(live), max_len), dtype=torch.bool, device=device)
    for row, i in enumerate(live):
        n = lens[i]
        keys[row, max_len - n :] = gather_kv(k_pool, block_tables[i], n).to(compute_dtype)
        values[row, max_len - n :] = gather_kv(v_pool, block_tables[i], n).to(compute_dtype)
        mask[row, max_len - n :] = True
    res = contiguous_attention(query[live].unsqueeze(1), keys, values, mask, max_len - 1)
    out[live] = res[:, 0]
    return out


def oracle_prefill(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    q_starts: torch.Tensor,
    q_lens: torch.Tensor,
    ctx_lens: torch.Tensor,
    compute_dtype: torch.dtype = torch.float32,
    seqs: list[int] | None = None,
    device: torch.device | str = "cpu",
) -> dict[int, torch.Tensor]:
    """Causal prefill over cached prefix + new tokens, one sequence at a time.

    Sequence b's rows ``query[q_starts[b] : q_starts[b] + q_lens[b]]`` attend
    keys ``[0, ctx_lens[b] + i]``: the reference's prefill bias with
    ``context_len = ctx_lens[b]`` and no padding (contiguous.py:136-169, :208),
    over the prefix + suffix K/V gathered through the block table.

    Returns {b: [q_lens[b], Hq, D] in compute_dtype} for the requested ``seqs``,
    computed on ``device`` (the CPU by default).
    """
    query = query.detach().to(device)
    k_pool = k_pool.detach().to(device)
    v_pool = v_pool.detach().to(device)
    block_tables = block_tables.detach().to(device)
    starts = q_starts.detach().cpu().tolist()
    qlens = q_lens.detach().cpu().tolist()
    ctxs = ctx_lens.detach().cpu().tolist()
    if seqs is None:
        seqs = list(range(len(starts)))
    result = {}
    for i in seqs:
        s, n, c = int(starts[i]), int(qlens[i]), int(ctxs[i])
        if n == 0:
            result[i] = torch.zeros((0, query.shape[1], query.shape[2]), dtype=compute_dtype,
                                    device=device)
            continue
        q = query[s : s + n].to(compute_dtype).unsqueeze(0)
        k = gather_kv(k_pool, block_tables[i], c + n).to(compute_dtype).unsqueeze(0)
        v = gather_kv(v_pool, block_tables[i], c + n).to(compute_dtype).unsqueeze(0)
        mask = torch.ones((1, c + n), dtype=torch.bool, device=device)
        result[i] = contiguous_attention(q, k, v, mask, c)[0]
    return result


# --------------------------------------------------------------------------- RoPE
def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Split-half rotation [a, b] -> [-b, a] (pagedserve/model/layers.py:49-59)."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_cos_sin(
    positions: torch.Tensor, head_dim: int, theta: float, dtype: torch.dtype
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of RotaryEmbedding (pagedserve/model/layers.py:91-116), computed on CPU.

    inv_freq = 1/theta**(arange(0, D, 2)/D) in fp32; freqs = pos * inv_freq;
    emb = cat(freqs, freqs); cos/sin in fp32, then cast to ``dtype``.
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = positions.float().unsqueeze(-1) * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_k(key: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """K half of apply_rotary (pagedserve/model/layers.py:62-77), in key's dtype.

    key [T, Hkv, D]; cos/sin [T, D] broadcast over heads. Each product and the
    sum round to the storage dtype, as torch's elementwise ops do.
    """
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (key * cos) + (rotate_half(key) * sin)


# --------------------------------------------------------------------------- cache writes
def oracle_append(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    positions: torch.Tensor | None = None,
    cos_sin_table: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """KV write through a slot mapping, on CPU copies of the pools.

    The write of ContiguousAttentionBackend.forward (contiguous.py:187-189) as a
    torch ``index_put`` at flat slots (block*bs + offset; -1 = skip). With
    ``positions``/``cos_sin_table`` K is first rotated as the reference does
    (layers.py:62-77) using the given table rows: cos = cat(c, c), sin = cat(s, s)
    where row p of the table is (c | s) — the duplicated halves of
    ``cat(freqs, freqs)`` (layers.py:115).
    """
    kp = k_pool.detach().cpu().clone()
    vp = v_pool.detach().cpu().clone()
    key = key.detach().cpu()
    value = value.detach().cpu()
    slots = slot_mapping.detach().cpu().long()
    if positions is not None:
        assert cos_sin_table is not None
        half = key.shape[-1] // 2
        rows = cos_sin_table.detach().cpu()[positions.detach().cpu().long()]
        c, s = rows[:, :half], rows[:, half:]
        key = _rotate_k(key, torch.cat((c, c), dim=-1), torch.cat((s, s), dim=-1))
    keep = slots >= 0
    slots = slots[keep]
    bs = kp.shape[2]
    blk, off = slots // bs, slots % bs
    kp[blk, :, off, :] = key[keep].to(kp.dtype)
    vp[blk, :, off, :] = value[keep].to(vp.dtype)
    return kp, vp


def oracle_copy_blocks(
    k_pool: torch.Tensor, v_pool: torch.Tensor, block_pairs: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """``pool[dst] = pool[src]`` per pair, on CPU copies.

    Copy-on-write of a shared block: the reference plans this (block manager
    fork/CoW) without implementing it, so the semantics are the plain block copy.
    Pools may carry a leading layer dimension.

    The pairs of one call are independent copies: a list whose destination
    repeats, or names another pair's source (a chain such as (a,b),(b,c)), has
    no single meaning once the copies run at the same time, so it is rejected
    with ValueError. Such a list is two calls, one after the other.
    """
    pairs = block_pairs.detach().cpu().tolist()
    dsts = [d for _, d in pairs]
    if len(set(dsts)) != len(dsts):
        raise ValueError("copy pairs: a destination block appears twice")
    for i, (_, d) in enumerate(pairs):
        if any(s == d for j, (s, _) in enumerate(pairs) if j != i):
            raise ValueError(f"copy pairs: destination block {d} is another pair's source")
    kp = k_pool.detach().cpu().clone()
    vp = v_pool.detach().cpu().clone()
    layered = kp.dim() == 5
    for src, dst in pairs:
        if layered:
            kp[:, dst] = kp[:, src]
            vp[:, dst] = vp[:, src]
        else:
            kp[dst] = kp[src]
            vp[dst] = vp[src]
    return kp, vp
