"""ps_paged_decode_noalloc: split-K decode with no device allocation at all.

Hosts such as a plugin inside a serving runtime, or a cgo/JNI/C engine whose
allocator owns every byte of device memory, can give this library only its
inputs and outputs; a latency-critical decode loop may also refuse
cudaMalloc/cudaFree because they can synchronise the device. For them the
library keeps the split-K partials in a 64 MiB array compiled into its device
image. This test calls that entry point through the C ABI (ctypes, raw
pointers) twice in a row with different batches — the second, larger call runs
on scratch still holding the first call's partials — and checks each result
bit for bit against ps_paged_decode with a caller-provided workspace (the same
plan, decode and combine kernels on the same inputs), and a sample of
sequences against the oracle within the attention tolerance. It lives in its
own file, collected last, so a failure here cannot hide the results of the
other tests.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_decode
from paged_serve_b200 import _lib, ops
from tests.gpu_util import assert_attention_close, random_pool, random_tables

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
HQ, HKV, D, BS = 32, 8, 128, 16
SPLIT = 512
WIDTH = 4096 // BS


def _noalloc(q, kp, vp, tables, ctx, split):
    lib = _lib.load()
    out = torch.empty_like(q)
    st = lib.ps_paged_decode_noalloc(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kp.data_ptr(), vp.data_ptr(),
        kp.shape[0], tables.data_ptr(), tables.stride(0), ctx.data_ptr(), q.shape[0], HQ, HKV, D,
        BS, tables.shape[1], D**-0.5, split, _lib.PS_DTYPE_BF16, None,
        torch.cuda.current_stream(DEV).cuda_stream,
    )
    _lib.check(st, "ps_paged_decode_noalloc")
    return out


def _with_workspace(q, kp, vp, tables, ctx, split):
    nbytes = ops.decode_workspace_bytes(q.shape[0], HQ, D, BS, tables.shape[1], split)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
    return ops.paged_decode(q, kp, vp, tables, ctx, D**-0.5, split, workspace=ws)


def _batch(seed: int, batch: int):
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 4097, (batch,), generator=gen).tolist()
    nb = sum((n + BS - 1) // BS for n in lens) + 11
    kp, vp = random_pool(nb, HKV, BS, D, torch.bfloat16, DEV, seed=seed)
    tables = random_tables(lens, BS, nb, seed=seed, width=WIDTH).to(DEV)
    q = (torch.randn((batch, HQ, D), generator=gen) * 0.5).to(torch.bfloat16).to(DEV)
    return q, kp, vp, tables, torch.tensor(lens, dtype=torch.int32, device=DEV)


def test_noalloc_decode_matches_the_workspace_entry_point_twice_in_a_row():
    # The larger batch second: its plan covers more (sequence, partition) units
    # than the first call left in the shared scratch.
    for seed, batch in ((22, 96), (21, 128)):
        q, kp, vp, tables, ctx = _batch(seed, batch)
        got = _noalloc(q, kp, vp, tables, ctx, SPLIT)
        ref = _with_workspace(q, kp, vp, tables, ctx, SPLIT)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"noalloc call seed {seed}: differs from the workspace path"
        pick = [0, batch // 3, batch - 1]
        want = oracle_decode(q[pick], kp, vp, tables[pick].cpu(), ctx[pick].cpu())
        assert_attention_close(got[pick], want, f"noalloc call seed {seed} vs oracle")


def test_noalloc_without_split_uses_no_scratch():
    q, kp, vp, tables, ctx = _batch(23, 16)
    got = _noalloc(q, kp, vp, tables, ctx, 0)
    ref = _with_workspace(q, kp, vp, tables, ctx, 0)
    assert torch.equal(got, ref)


def test_requests_beyond_the_scratch_are_rejected():
    lib = _lib.load()
    need = lib.ps_paged_decode_workspace_bytes(4096, HQ, D, BS, WIDTH, SPLIT)
    assert need > 64 << 20
    st = lib.ps_paged_decode_noalloc(16, HQ * D, 16, HQ * D, 16, 16, 1 << 20, 16, WIDTH, 16,
                                     4096, HQ, HKV, D, BS, WIDTH, 0.1, SPLIT,
                                     _lib.PS_DTYPE_BF16, None, None)
    assert st == _lib.PS_ERR_INVALID
    assert "built-in scratch" in lib.ps_last_error_string().decode()


def test_invalid_arguments_report_their_own_error_first():
    """A batch too large for one launch is reported as such, not as a scratch overflow."""
    lib = _lib.load()
    st = lib.ps_paged_decode_noalloc(16, HQ * D, 16, HQ * D, 16, 16, 1 << 20, 16, WIDTH, 16,
                                     70000, HQ, HKV, D, BS, WIDTH, 0.1, SPLIT,
                                     _lib.PS_DTYPE_BF16, None, None)
    assert st == _lib.PS_ERR_INVALID
    msg = lib.ps_last_error_string().decode()
    assert "too many sequences" in msg and "scratch" not in msg
