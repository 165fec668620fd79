"""GPU failure path without a GPU fault: a bounded wait that runs out.

Every kernel waits on mbarriers with the same poll bound and, when it runs out,
records PS_DEVERR_TIMEOUT and leaves instead of hanging. Here a wait on an
mbarrier that nothing arrives at makes that bound run out; the status must come
back and the context must stay usable for the next launch.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle_decode
from paged_serve_b200 import _lib, ops
from tests.gpu_util import assert_attention_close, random_pool, random_tables

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_bounded_wait_times_out_reports_and_context_survives():
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ops.selftest_wait_timeout(err)
    e1.record()
    torch.cuda.synchronize()
    assert int(err.item()) == _lib.PS_DEVERR_TIMEOUT
    ms = e0.elapsed_time(e1)
    print(f"bounded wait gave up after {ms:.1f} ms")
    assert 500 < ms < 5_000  # the bound is one second of failed polls

    # the same context runs the next launch normally
    lens = [5, 300, 17]
    kp, vp = random_pool(64, 2, 16, 128, torch.bfloat16, DEV, seed=71)
    tables = random_tables(lens, 16, 64, seed=72)
    q = (torch.randn((3, 8, 128), generator=torch.Generator().manual_seed(73)) * 0.5).to(
        torch.bfloat16).to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32)
    err.zero_()
    out = ops.paged_decode(q, kp, vp, tables.to(DEV), ctx.to(DEV), 128 ** -0.5, 0,
                           device_error=err)
    assert int(err.item()) == 0
    assert_attention_close(out, oracle_decode(q, kp, vp, tables, ctx), "after timeout")
