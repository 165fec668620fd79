"""Multi-process host logic on CPU ``gloo`` ranks (world size 2).

The GPU bench shards sequences across ranks with no data-path collective and
uses collectives only to combine timings and to verify outputs. These tests run
the same host steps on CPU ranks: every rank derives its own LPT shard from the
shared seed, the shards partition the global batch, max-over-ranks timing is a
MAX all-reduce, each rank checks its share against the oracle and the flags are
all-gathered; and a rank that leaves early makes the survivor's next collective
fail within the process group's timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _init(rank, world, port)
    from oracle import oracle_decode
    from paged_serve_b200.workloads import decode_workload

    wl = decode_workload("llama8b", seed=0, rank=rank, world=world, weak=True, batch=16)
    ids = wl.seq_ids
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([ids.numel()]))
    gathered = [torch.zeros(int(s.item()), dtype=torch.int64) for s in sizes]
    dist.all_gather(gathered, ids)
    # max-over-ranks timing, as bench.py reports it
    t = torch.tensor([float(rank + 1) * 1.5], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    # each rank verifies a tiny share of its own work on the oracle, flags are gathered
    g = torch.Generator().manual_seed(rank)
    s = wl.spec
    lens = [3, 17]
    pool = torch.randn((4, s.num_kv_heads, 16, s.head_dim), generator=g)
    tables = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32)
    q = torch.randn((2, s.num_q_heads, s.head_dim), generator=g)
    out = oracle_decode(q, pool, pool, tables, torch.tensor(lens, dtype=torch.int32))
    ok = torch.tensor([1.0 if bool(torch.isfinite(out).all()) else 0.0, float(out.sum())])
    flags = [torch.zeros(2) for _ in range(world)]
    dist.all_gather(flags, ok)
    if rank == 0:
        torch.save({"ids": [x.tolist() for x in gathered], "tmax": float(t.item()),
                    "flags": [f.tolist() for f in flags],
                    "tokens": [int(decode_workload("llama8b", seed=0, rank=r, world=world,
                                                   weak=True, batch=16).total_tokens)
                               for r in range(world)]},
                   os.path.join(out_dir, "result.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_shard_time_and_verify(tmp_path):
    world = 2
    mp.start_processes(_shard_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    res = torch.load(tmp_path / "result.pt")
    allids = sorted(res["ids"][0] + res["ids"][1])
    assert allids == list(range(16 * world)), "shards must partition the global batch"
    assert not set(res["ids"][0]) & set(res["ids"][1])
    assert res["tmax"] == pytest.approx(3.0)
    assert all(f[0] == 1.0 for f in res["flags"])
    a, b = res["tokens"]
    assert abs(a - b) <= 4096, "LPT keeps the ranks' token loads within one sequence"


def _failing_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _init(rank, world, port, timeout_s=5.0)
    dist.barrier()  # both ranks are up
    if rank == 1:
        # leaves between steps, with nothing in flight, without telling anyone
        os._exit(0)
    err = ""
    try:
        t = torch.ones(1)
        dist.all_reduce(t)  # the next step's collective: the peer is gone
    except Exception as e:  # noqa: BLE001 - any failure type is a detection
        err = type(e).__name__ + ": " + str(e)[:200]
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(err or "NO ERROR")
    os._exit(0)


def test_lost_rank_is_detected_by_the_survivor(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung instead of detecting the lost peer")
    msg = (tmp_path / "rank0.txt").read_text()
    assert msg != "NO ERROR", "the survivor's collective must fail, not succeed"
