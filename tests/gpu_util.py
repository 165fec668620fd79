"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import torch

# Tolerance for bf16/fp16 attention outputs against the fp32 oracle: an element
# passes when |got - ref| <= ATOL + RTOL * |ref| (max-abs 2e-3, relative 1e-2).
ATOL = 2e-3
RTOL = 1e-2


def assert_attention_close(got: torch.Tensor, ref: torch.Tensor, what: str = "") -> None:
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = (got - ref).abs()
    bound = ATOL + RTOL * ref.abs()
    bad = err > bound
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(
            f"{what}: {int(bad.sum())} elements outside |d| <= {ATOL} + {RTOL}|ref|; "
            f"max abs err {float(err.max()):.3e}; first at {idx}: got "
            f"{float(got[tuple(idx)]):.6f} ref {float(ref[tuple(idx)]):.6f}"
        )


def random_pool(num_blocks: int, hkv: int, bs: int, d: int, dtype, device, seed: int,
                scale: float = 0.5):
    gen = torch.Generator(device=device).manual_seed(seed)
    k = torch.empty((num_blocks, hkv, bs, d), dtype=dtype, device=device)
    v = torch.empty_like(k)
    k.normal_(0.0, scale, generator=gen)
    v.normal_(0.0, scale, generator=gen)
    return k, v


def random_tables(lens: list[int], bs: int, num_blocks: int, seed: int, width: int | None = None):
    gen = torch.Generator().manual_seed(seed)
    need = [(n + bs - 1) // bs for n in lens]
    perm = torch.randperm(num_blocks, generator=gen)
    width = width or max(need + [1])
    tables = torch.zeros((len(lens), width), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[pos : pos + n].to(torch.int32)
        pos += n
    assert pos <= num_blocks
    return tables


def oracle_decode_on_device(query, k_pool, v_pool, block_tables, ctx_lens,
                            token_budget: int = 65536) -> torch.Tensor:
    """The oracle's decode steps for a whole batch, run on the pools' device in fp32.

    Sequences are grouped (shortest first) into chunks of at most ``token_budget``
    padded keys, so a full-size batch is checked in seconds without holding its
    dense, GQA-expanded copy at once. Returns [B, Hq, D] fp32 on that device.
    """
    from oracle import oracle_decode

    dev = k_pool.device
    lens = [int(x) for x in ctx_lens.detach().cpu().tolist()]
    out = torch.zeros(query.shape, dtype=torch.float32, device=dev)
    order = sorted(range(len(lens)), key=lambda i: lens[i])
    i = 0
    while i < len(order):
        chunk = [order[i]]
        i += 1
        while i < len(order) and (len(chunk) + 1) * max(1, lens[order[i]]) <= token_budget:
            chunk.append(order[i])
            i += 1
        idx = torch.tensor(chunk, device=dev)
        out[idx] = oracle_decode(query[idx], k_pool, v_pool, block_tables.to(dev)[idx],
                                 torch.tensor([lens[j] for j in chunk]), device=dev)
    return out
