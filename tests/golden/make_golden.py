"""Generate the golden fixtures in this directory by running the reference itself.

Runs Vivek-Chaudhari30/Paged_Serve's own ``ContiguousAttentionBackend``,
``RotaryEmbedding`` and ``apply_rotary`` (pure PyTorch, CPU) on seeded inputs
and stores inputs + outputs as small ``.pt`` files. The reference cannot be
installed where the GPU tests run, so the fixtures carry its answers there.

Usage (needs a checkout of the reference project, named by --reference or by
the PAGEDSERVE_REFERENCE environment variable):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

Every fixture records ``generator`` (this file) and the reference call it came from.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from paged_serve_b200.workloads import assign_blocks, decode_workload  # noqa: E402


def _model_config(ModelConfig, hq: int, hkv: int, d: int, theta: float = 10000.0):
    return ModelConfig(
        name="golden", num_layers=1, hidden_size=hq * d, num_q_heads=hq, num_kv_heads=hkv,
        head_dim=d, intermediate_size=4 * hq * d, vocab_size=32, rms_norm_eps=1e-6,
        rope_theta=theta, max_position_embeddings=65536, tie_word_embeddings=False,
        attention_bias=False,
    )


def _pool_from_seqs(keys: list[torch.Tensor], tables: torch.Tensor, num_blocks: int, bs: int):
    """Scatter per-sequence [n, Hkv, D] tensors into a zeroed [num_blocks, Hkv, bs, D] pool."""
    hkv, d = keys[0].shape[1:]
    pool = torch.zeros((num_blocks, hkv, bs, d), dtype=keys[0].dtype)
    for i, k in enumerate(keys):
        n = k.shape[0]
        for j in range((n + bs - 1) // bs):
            chunk = k[j * bs : (j + 1) * bs]
            pool[int(tables[i, j]), :, : chunk.shape[0]] = chunk.transpose(0, 1)
    return pool


def ref_decode(ref, hq, hkv, d, q, keys, values, compute_dtype):
    """The reference's decode step on left-padded sequences; returns [B, Hq, D].

    Sequence b's first ctx_b - 1 tokens are written into the dense cache as a
    previous step would have; the decode step then writes token ctx_b - 1 and
    attends (ContiguousAttentionBackend.begin_step + forward).
    """
    backend_mod, contiguous_mod, config_mod = ref
    cfg = _model_config(config_mod.ModelConfig, hq, hkv, d)
    lens = [k.shape[0] for k in keys]
    max_len = max(lens)
    b = len(keys)
    be = contiguous_mod.ContiguousAttentionBackend(cfg, device=torch.device("cpu"),
                                                    dtype=compute_dtype)
    be.allocate(num_seq_slots=b, max_seq_len=max_len)
    mask = torch.zeros((b, max_len), dtype=torch.bool)
    for i, (k, v) in enumerate(zip(keys, values, strict=True)):
        n = k.shape[0]
        be.kv_cache[0, 0, i, max_len - n : max_len - 1] = k[:-1].to(compute_dtype)
        be.kv_cache[0, 1, i, max_len - n : max_len - 1] = v[:-1].to(compute_dtype)
        mask[i, max_len - n :] = True
    step = backend_mod.StepInput(query_len=1, context_len=max_len - 1,
                                 seq_lens=torch.tensor(lens, dtype=torch.int32),
                                 padding_mask=mask, is_prefill=False)
    md = be.begin_step(step)
    k_new = torch.stack([k[-1] for k in keys]).unsqueeze(1).to(compute_dtype)
    v_new = torch.stack([v[-1] for v in values]).unsqueeze(1).to(compute_dtype)
    out = be.forward(0, q.unsqueeze(1).to(compute_dtype), k_new, v_new, md)
    return out[:, 0]


def ref_prefill(ref, hq, hkv, d, q, keys, values, prefix, compute_dtype):
    """One sequence: a first forward caches the prefix, a second runs the suffix."""
    backend_mod, contiguous_mod, config_mod = ref
    cfg = _model_config(config_mod.ModelConfig, hq, hkv, d)
    n_new = q.shape[0]
    total = prefix + n_new
    be = contiguous_mod.ContiguousAttentionBackend(cfg, device=torch.device("cpu"),
                                                    dtype=compute_dtype)
    be.allocate(num_seq_slots=1, max_seq_len=total)
    k = keys.to(compute_dtype).unsqueeze(0)
    v = values.to(compute_dtype).unsqueeze(0)
    if prefix:
        step = backend_mod.StepInput(query_len=prefix, context_len=0,
                                     seq_lens=torch.tensor([prefix], dtype=torch.int32),
                                     padding_mask=torch.ones((1, prefix), dtype=torch.bool),
                                     is_prefill=True)
        md = be.begin_step(step)
        dummy_q = torch.zeros((1, prefix, hq, d), dtype=compute_dtype)
        be.forward(0, dummy_q, k[:, :prefix], v[:, :prefix], md)
    step = backend_mod.StepInput(query_len=n_new, context_len=prefix,
                                 seq_lens=torch.tensor([total], dtype=torch.int32),
                                 padding_mask=torch.ones((1, total), dtype=torch.bool),
                                 is_prefill=True)
    md = be.begin_step(step)
    out = be.forward(0, q.to(compute_dtype).unsqueeze(0), k[:, prefix:], v[:, prefix:], md)
    return out[0]


def make_decode_case(ref, name, hq, hkv, d, lens, in_dtype, compute_dtype, seed, pool_blocks):
    """Values ~ 0.5*N(0,1), the distribution of the decode workloads."""
    gen = torch.Generator().manual_seed(seed)
    bs = 16
    keys = [(0.5 * torch.randn((n, hkv, d), generator=gen)).to(in_dtype) for n in lens]
    values = [(0.5 * torch.randn((n, hkv, d), generator=gen)).to(in_dtype) for n in lens]
    q = (0.5 * torch.randn((len(lens), hq, d), generator=gen)).to(in_dtype)
    bps = [(n + bs - 1) // bs for n in lens]
    tables = assign_blocks(bps, pool_blocks, gen)
    out = ref_decode(ref, hq, hkv, d, q, keys, values, compute_dtype)
    return {
        "name": name, "generator": "tests/golden/make_golden.py",
        "reference_call": "ContiguousAttentionBackend.begin_step+forward (decode, left-padded)",
        "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d, "block_size": bs,
        "num_blocks": pool_blocks, "ctx_lens": torch.tensor(lens, dtype=torch.int32),
        "block_tables": tables, "query": q, "keys": torch.cat(keys), "values": torch.cat(values),
        "expected": out.to(torch.float32), "compute_dtype": str(compute_dtype),
    }


def make_prefill_case(ref, name, hq, hkv, d, prefixes, news, in_dtype, compute_dtype, seed,
                      pool_blocks):
    """Values ~ 0.5*N(0,1), the distribution of the prefix-prefill workload."""
    gen = torch.Generator().manual_seed(seed)
    bs = 16
    keys, values, qs, outs = [], [], [], []
    for p, n in zip(prefixes, news, strict=True):
        k = (0.5 * torch.randn((p + n, hkv, d), generator=gen)).to(in_dtype)
        v = (0.5 * torch.randn((p + n, hkv, d), generator=gen)).to(in_dtype)
        q = (0.5 * torch.randn((n, hq, d), generator=gen)).to(in_dtype)
        outs.append(ref_prefill(ref, hq, hkv, d, q, k, v, p, compute_dtype))
        keys.append(k)
        values.append(v)
        qs.append(q)
    bps = [(p + n + bs - 1) // bs for p, n in zip(prefixes, news, strict=True)]
    tables = assign_blocks(bps, pool_blocks, gen)
    return {
        "name": name, "generator": "tests/golden/make_golden.py",
        "reference_call": "ContiguousAttentionBackend prefill of prefix, then of new tokens",
        "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d, "block_size": bs,
        "num_blocks": pool_blocks, "prefix_lens": torch.tensor(prefixes, dtype=torch.int32),
        "q_lens": torch.tensor(news, dtype=torch.int32), "block_tables": tables,
        "query": torch.cat(qs), "keys": torch.cat(keys), "values": torch.cat(values),
        "expected": torch.cat(outs).to(torch.float32), "compute_dtype": str(compute_dtype),
    }


def make_rope_case(layers_mod, name, t, hkv, d, theta, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn((t, hkv, d), generator=gen).to(dtype)
    positions = torch.cat([torch.arange(0, t // 2), torch.randint(0, 32768, (t - t // 2,),
                                                                  generator=gen)])
    rot = layers_mod.RotaryEmbedding(head_dim=d, theta=theta, device=torch.device("cpu"))
    cos, sin = rot(positions.unsqueeze(0), dtype)
    q_dummy = torch.zeros((1, t, 1, d), dtype=dtype)
    _, k_rot = layers_mod.apply_rotary(q_dummy, k.unsqueeze(0), cos, sin)
    return {
        "name": name, "generator": "tests/golden/make_golden.py",
        "reference_call": "RotaryEmbedding(head_dim, theta).forward + apply_rotary (K)",
        "theta": theta, "key": k, "positions": positions, "cos": cos[0], "sin": sin[0],
        "expected": k_rot[0],
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PAGEDSERVE_REFERENCE"),
                    help="reference checkout (default: $PAGEDSERVE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or PAGEDSERVE_REFERENCE")
    sys.path.insert(0, args.reference)
    import pagedserve.attention.backend as backend_mod
    import pagedserve.attention.contiguous as contiguous_mod
    import pagedserve.config as config_mod
    import pagedserve.model.layers as layers_mod

    ref = (backend_mod, contiguous_mod, config_mod)
    torch.manual_seed(0)

    # Workload "tiny": the host plumbing case, fp32 end to end, its own seeded draw.
    wl = decode_workload("tiny", seed=0)
    gen = torch.Generator().manual_seed(0)
    lens = wl.ctx_lens.tolist()
    keys = [torch.randn((n, 2, 64), generator=gen) for n in lens]
    values = [torch.randn((n, 2, 64), generator=gen) for n in lens]
    q = torch.randn((4, 8, 64), generator=gen)
    out = ref_decode(ref, 8, 2, 64, q, keys, values, torch.float32)
    torch.save({
        "name": "tiny_decode", "generator": "tests/golden/make_golden.py",
        "reference_call": "ContiguousAttentionBackend.begin_step+forward (decode, left-padded)",
        "num_q_heads": 8, "num_kv_heads": 2, "head_dim": 64, "block_size": 16,
        "num_blocks": wl.num_blocks, "ctx_lens": wl.ctx_lens, "block_tables": wl.block_tables,
        "query": q, "keys": torch.cat(keys), "values": torch.cat(values), "expected": out,
        "compute_dtype": "torch.float32",
    }, HERE / "tiny_decode.pt")

    # bf16 decode, Llama-3 head geometry (GQA 4), block-boundary lengths.
    torch.save(make_decode_case(ref, "decode_bf16_gqa4", 32, 8, 128, [1, 15, 16, 17, 130],
                                torch.bfloat16, torch.float32, 1, 64),
               HERE / "decode_bf16_gqa4.pt")
    # bf16 decode, Qwen2.5-0.5B head geometry (GQA 7, head_dim 64).
    torch.save(make_decode_case(ref, "decode_bf16_gqa7", 14, 2, 64, [33, 250, 513],
                                torch.bfloat16, torch.float32, 2, 80),
               HERE / "decode_bf16_gqa7.pt")
    # bf16 causal prefill over cached prefixes (0, mid-block, block-aligned).
    torch.save(make_prefill_case(ref, "prefill_bf16_gqa4", 8, 2, 128, [0, 37, 64], [5, 40, 16],
                                 torch.bfloat16, torch.float32, 3, 24),
               HERE / "prefill_bf16_gqa4.pt")
    # RoPE on K: reference cos/sin and rotation in bf16 (theta of Llama-3) and fp16.
    torch.save(make_rope_case(layers_mod, "rope_bf16", 64, 2, 128, 500000.0, torch.bfloat16, 4),
               HERE / "rope_bf16.pt")
    torch.save(make_rope_case(layers_mod, "rope_f16", 32, 2, 64, 10000.0, torch.float16, 5),
               HERE / "rope_f16.pt")
    for p in sorted(HERE.glob("*.pt")):
        print(f"{p.name}: {p.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
