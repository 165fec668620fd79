"""Benchmark of the paged KV hot path on B200 (one JSON line on rank 0).

Default workload (``llama8b``): Llama-3-8B-shaped decode, all 32 layers — per
layer one paged decode launch that also appends the step's new token —
256 sequences per GPU with ctx ~ U[512, 4096], bf16, block size 16, random
synthetic KV (seeded). A step = the 32 layers. ``value`` = decode tokens/s
summed over all GPUs (each rank owns its own token-balanced share of a
256*N-sequence global batch: weak scaling, no collective on the data path);
``roofline`` = achieved HBM GB/s of one decode layer (algorithmic bytes /
CUDA-event time) against the measured copy bandwidth, and against the read
ceiling of a read-only stream measured in the same run; ``e2e`` = the same
tokens/s through ``PagedCudaBackend`` with every step's inputs copied from
pinned host memory and every layer's output copied back, inside the timed
region.

The default line also carries the other hot-path workloads as sub-results,
each with its own roofline, clocks, oracle check and CPU baseline:
``append`` (fused RoPE append, 16640 tokens x 32 per-layer calls),
``prefill`` (prefix-cached prefill with copy-on-write, one layer) and
``llama70b`` (long-context skewed decode, 80 layers: one 512-sequence batch
sharded over the GPUs by greedy token balance — strong scaling — with the
per-rank token loads and step times) and ``mixed`` (continuous batching with
chunked prefill through the block manager). ``--headline-only`` skips them;
``--workload`` runs one of them (or ``continuous`` / ``swap``) on its own.

``--impl reference`` times the reference's own algorithm for the same workload
on the host CPU cores (the CPU restatement of its contiguous attention path in
``oracle/``) on a bounded sample of each step, extrapolated linearly to the
full step (labelled ``extrapolated``).

Launch: ``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 under
``torch.distributed.run`` (one process per GPU, RANK/LOCAL_RANK/WORLD_SIZE).
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode paged-attn HBM GB/s (% of peak) and decode tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 * 2**20


# ----------------------------------------------------------------------------- helpers
def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str) -> float | None:
    """Per-launch DRAM bytes of a kernel from a committed ncu summary, if present."""
    p = ROOT / "profiles" / f"{name}.traffic.json"
    if not p.exists():
        return None
    try:
        return float(json.loads(p.read_text())["dram_bytes_per_launch"])
    except (KeyError, ValueError):
        return None


class ClockSampler:
    """SM clock and clock-event reasons sampled every 20 ms while the timed region runs.

    Reads NVML (the library behind nvidia-smi) from a background thread; only
    samples taken after ``start()`` (called as the timed region begins) and
    before the context exits (after the closing synchronize) are kept, so idle
    lead-in samples never enter the median. Falls back to nvidia-smi at 100 ms
    when NVML is unavailable.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.02

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.nvml = None
        self.handle = None
        self.rows: list[tuple[float, float, list[str]]] = []
        self.recording = False
        self.stop = False
        self.thread = None
        self.max_mhz = None
        self.power_w: list[float] = []

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            handle = pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:  # older drivers/torch: fall back to the CUDA index
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
        return pynvml, handle

    def _sample_loop(self):
        nv = self.nvml
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
                 "hw_power_brake": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown}
        while not self.stop:
            if self.recording:
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                    self.rows.append((mhz, self.max_mhz, [n for n, b in names.items() if bits & b]))
                    self.power_w.append(nv.nvmlDeviceGetPowerUsage(self.handle) / 1e3)
                except Exception:
                    pass
            time.sleep(self.PERIOD_S)

    def __enter__(self):
        import threading

        try:
            self.nvml, self.handle = self._nvml_handle()
            self.max_mhz = float(self.nvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                     self.nvml.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._sample_loop, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def start(self) -> None:
        """Called as the timed region begins."""
        self.recording = True

    def __exit__(self, *exc):
        self.recording = False
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=1.0)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        rows = self.rows
        if self.nvml is None:
            if self.proc is None or self.file is None:
                return None
            rows = []
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in Path(self.file.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]),
                                 [names[i] for i in range(4) if parts[5 + i] == "Active"]))
                except ValueError:
                    continue
            os.unlink(self.file.name)
        if not rows:
            return None
        reasons = sorted({r for _, _, rs in rows for r in rs})
        out = {"sm_mhz": statistics.median(r[0] for r in rows), "sm_min_mhz": min(r[0] for r in rows),
               "sm_max_mhz": rows[0][1], "reasons": reasons, "samples": len(rows),
               "power_cap_fraction": sum("sw_power_cap" in rs for _, _, rs in rows) / len(rows),
               "source": "nvml, 20 ms, timed region only" if self.nvml is not None
               else "nvidia-smi, 100 ms"}
        if self.power_w:
            out["power_w_median"] = statistics.median(self.power_w)
        return out


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


def gather_objects(obj, world: int) -> list:
    """Every rank's ``obj`` (small, picklable), in rank order, on every rank."""
    if world == 1:
        return [obj]
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def read_ceiling(dev: torch.device, gib: int = 4, reps: int = 10) -> dict:
    """HBM read bandwidth of ps_stream_read over a buffer far larger than L2.

    The copy peak (MEASURED_PEAKS.json) moves every byte both ways; a kernel
    that mostly reads, like the paged decode, is bounded by this instead. Two
    read methods are timed (bulk asynchronous copies into shared memory, the
    decode's path; and 16-byte loads); the ceiling is the faster.
    """
    from paged_serve_b200 import _lib, ops

    buf = torch.ones(gib << 28, dtype=torch.int32, device=dev)  # gib GiB
    acc = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    nbytes = buf.numel() * 4
    out = {}
    for name, method in (("bulk_copies", _lib.PS_STREAM_BULK), ("loads", _lib.PS_STREAM_LOADS)):
        times = []
        for i in range(reps + 2):
            a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ops.stream_read(buf, acc, method, err)
            z.record(stream)
            torch.cuda.synchronize(dev)
            if i >= 2:
                times.append(a.elapsed_time(z))
        out[name] = {"gbs": nbytes / (min(times) / 1e3) / 1e9,
                     "median_gbs": nbytes / (statistics.median(times) / 1e3) / 1e9}
    if int(err.item()):
        raise RuntimeError("read stream: a bounded wait ran out")
    del buf
    best = max(out.values(), key=lambda r: r["gbs"])
    return {"gbs": best["gbs"], "methods": out, "bytes": nbytes,
            "kernel": "ps_stream_read: bulk_copies = 8 KB cp.async.bulk chunks into per-warp "
                      "2-stage shared-memory rings, 3 CTAs x 4 warps per SM; loads = 16-byte "
                      "evict-first loads, 8 in flight per thread, 8 CTAs x 256 threads per SM",
            "how": f"best of {reps} CUDA-event-timed passes over {gib} GiB per method"}


def verify_decode_full_batch(q, k_pool, v_pool, tables, ctx, got, token_budget: int = 65536):
    """Every sequence of one decode layer against the oracle's steps run on the GPU in fp32.

    Sequences go through ``oracle_decode(device=...)`` in chunks of about
    ``token_budget`` keys. Returns (all within tolerance, worst |err| / bound).
    """
    from oracle import oracle_decode

    dev = q.device
    lens = ctx.tolist() if not isinstance(ctx, list) else ctx
    order = sorted(range(len(lens)), key=lambda i: lens[i])
    worst = 0.0
    i = 0
    while i < len(order):
        chunk = [order[i]]
        i += 1
        while i < len(order) and (len(chunk) + 1) * lens[order[i]] <= token_budget:
            chunk.append(order[i])
            i += 1
        idx = torch.tensor(chunk, device=dev)
        ref = oracle_decode(q[idx], k_pool, v_pool, tables[idx], torch.tensor(
            [lens[j] for j in chunk]), device=dev)
        err = (got[idx].float() - ref).abs()
        bound = 2e-3 + 1e-2 * ref.abs()
        worst = max(worst, float((err / bound).max()))
    return worst <= 1.0, worst


def timed_region(run_step, steps: int, warmup: int, world: int, gpu_index: int):
    """W warm-up steps, then exactly K steps between barrier+sync; device ms (this rank)."""
    for _ in range(warmup):
        run_step(False)
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_index) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        clocks.start()
        start.record(stream)
        for _ in range(steps):
            run_step(True)
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    return start.elapsed_time(end), clocks.summary()


# ----------------------------------------------------------------------------- decode
def cpu_decode_sample(wl, seqs: int, reps: int) -> dict:
    """Time the reference's contiguous decode path (the oracle restatement) on the CPU.

    Sample: one layer of ``seqs`` sequences of the workload's draw, fp32, with
    the dense left-padded cache already holding every earlier token — the
    reference's steady state (contiguous.py:113-209): build the mask, write the
    step's K/V slice, read the prefix, expand GQA, SDPA. Returns seconds per
    sample and the extrapolated tokens/s of the full workload on these cores.
    """
    from oracle import contiguous_attention

    s = wl.spec
    idx = torch.linspace(0, wl.batch - 1, seqs).round().long()
    lens = wl.ctx_lens[idx].tolist()
    max_len = max(lens)
    gen = torch.Generator().manual_seed(0)
    keys = torch.zeros((seqs, max_len, s.num_kv_heads, s.head_dim))
    values = torch.zeros_like(keys)
    mask = torch.zeros((seqs, max_len), dtype=torch.bool)
    for i, n in enumerate(lens):
        keys[i, max_len - n :] = torch.randn((n, s.num_kv_heads, s.head_dim), generator=gen) * 0.5
        values[i, max_len - n :] = torch.randn((n, s.num_kv_heads, s.head_dim), generator=gen) * .5
        mask[i, max_len - n :] = True
    q = torch.randn((seqs, 1, s.num_q_heads, s.head_dim), generator=gen) * 0.5
    k_new = torch.randn((seqs, 1, s.num_kv_heads, s.head_dim), generator=gen) * 0.5
    v_new = torch.randn_like(k_new)

    def one():
        keys[:, max_len - 1 : max_len] = k_new
        values[:, max_len - 1 : max_len] = v_new
        return contiguous_attention(q, keys, values, mask, max_len - 1)

    one()
    t0 = time.perf_counter()
    for _ in range(reps):
        one()
    per = (time.perf_counter() - t0) / reps
    sample_tokens = sum(lens)
    # extrapolate by KV tokens (the work is linear in them) to the full step
    full_step = per * (wl.total_tokens / sample_tokens) * s.num_layers
    return {"seconds_per_sample": per, "tokens_per_s": wl.batch / full_step,
            "sample_fraction": sample_tokens / (wl.total_tokens * s.num_layers),
            "sample": f"1 of {s.num_layers} layers x {seqs} of {wl.batch} sequences "
                      f"({sample_tokens} KV tokens, fp32, dense left-padded cache), "
                      f"{reps} reps; extrapolated linearly in KV tokens to the full step",
            "cores": torch.get_num_threads()}


def cpu_append_sample(wl, reps: int = 2) -> dict:
    """Time the reference's KV write with RoPE (the oracle: reference RoPE ops in
    the pool dtype, then an index_put through the slots) for one layer on the CPU.

    The touched blocks are renumbered into a compact pool (same slots within each
    block), so the sample does not allocate the full multi-GB pool on the host.
    """
    from oracle import oracle_append
    from paged_serve_b200.rope import cos_sin_table

    g = torch.Generator().manual_seed(0)
    slots = wl.slot_mapping.clone()
    blocks = torch.unique(slots // wl.block_size)
    remap = torch.full((wl.num_blocks,), -1, dtype=torch.int64)
    remap[blocks] = torch.arange(blocks.numel())
    compact = remap[slots // wl.block_size] * wl.block_size + slots % wl.block_size
    shape = (blocks.numel(), wl.num_kv_heads, wl.block_size, wl.head_dim)
    kp = torch.zeros(shape, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    key = torch.randn((wl.num_tokens, wl.num_kv_heads, wl.head_dim), generator=g).to(torch.bfloat16)
    value = torch.randn_like(key.float()).to(torch.bfloat16)
    table = cos_sin_table(wl.head_dim, wl.rope_theta, int(wl.positions.max()) + 1, torch.bfloat16,
                          torch.device("cpu"))
    oracle_append(kp, vp, key, value, compact, wl.positions, table)
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle_append(kp, vp, key, value, compact, wl.positions, table)
    per = (time.perf_counter() - t0) / reps
    return {"value": wl.num_tokens / per, "unit": "token-layers/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"one layer: {wl.num_tokens} tokens, reference RoPE in bf16 + index_put into "
                      f"a compact {blocks.numel()}-block pool, {reps} reps"}


def cpu_prefix_sample(wl, k_pool, v_pool, q, seqs: int = 4) -> dict:
    """Time the reference's contiguous prefill (the oracle, fp32) for a few sequences
    of the prefix workload on the CPU and extrapolate to all of them."""
    from oracle import oracle_prefill

    kp, vp, qc = k_pool.cpu(), v_pool.cpu(), q.cpu()
    pick = torch.linspace(0, wl.batch - 1, seqs).round().long().tolist()
    args = (qc, kp, vp, wl.block_tables, wl.q_starts, wl.q_lens, wl.prefix_lens)
    oracle_prefill(*args, seqs=pick[:1])
    t0 = time.perf_counter()
    oracle_prefill(*args, seqs=pick)
    per_seq = (time.perf_counter() - t0) / seqs
    return {"value": wl.total_q / (per_seq * wl.batch), "unit": "tokens/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{seqs} of {wl.batch} sequences (fp32 contiguous attention over prefix + "
                      f"causal suffix), extrapolated to all {wl.batch}"}


def bench_decode(args, rank: int, world: int, local_rank: int) -> dict:
    from paged_serve_b200 import ops
    from paged_serve_b200.backend import PagedCudaBackend
    from paged_serve_b200.config import ModelConfig
    from paged_serve_b200.interface import StepInput
    from paged_serve_b200.workloads import decode_workload

    dev = torch.device("cuda", local_rank)
    weak = args.scaling == "weak"
    wl = decode_workload(args.workload, seed=args.seed, rank=rank, world=world, weak=weak,
                         batch=args.batch)
    s = wl.spec
    layers = args.layers or s.num_layers
    b, hq, hkv, d = wl.batch, s.num_q_heads, s.num_kv_heads, s.head_dim
    dtype = torch.bfloat16
    elem = 2
    per_layer_pool = 2 * wl.num_blocks * hkv * s.block_size * d * elem
    free, _ = torch.cuda.mem_get_info(dev)
    budget = int(free * 0.80) - (256 << 20)
    pools = max(1, min(layers, budget // per_layer_pool))
    split = args.split_tokens
    max_len = wl.block_tables.shape[1] * s.block_size
    model = ModelConfig(s.name, num_layers=pools, num_q_heads=hq, num_kv_heads=hkv, head_dim=d,
                        rope_theta=s.rope_theta)
    backend = PagedCudaBackend(model, device=dev, dtype=dtype, block_size=s.block_size,
                               num_blocks=wl.num_blocks, split_tokens=split)
    backend.allocate(num_seq_slots=b, max_seq_len=max_len)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
    backend.k_cache.normal_(0.0, s.value_scale, generator=gen)
    backend.v_cache.normal_(0.0, s.value_scale, generator=gen)

    tables = wl.block_tables.to(dev)
    ctx = wl.ctx_lens.to(dev)
    pos = (wl.ctx_lens.long() - 1)
    slots = (wl.block_tables.long().gather(1, (pos // s.block_size).view(-1, 1)).view(-1)
             * s.block_size + pos % s.block_size).to(dev)
    nq = min(layers, 32)  # distinct per-layer inputs kept resident, cycled
    q = torch.empty((nq, b, hq, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    k_new = torch.empty((nq, b, hkv, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    out = torch.empty((nq, b, hq, d), dtype=dtype, device=dev)
    ws = backend._workspace
    err = backend.device_error
    scale = 1.0 / math.sqrt(d)
    stream = torch.cuda.current_stream(dev)
    dec_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    order = torch.empty_like(ctx)

    def run_step(record: bool):
        ops.decode_order(ctx, out=order)  # one longest-first launch order per step
        if split:  # and one split-K plan per step, shared by every layer
            ops.decode_plan(ctx, ws, hq, d, s.block_size, tables.shape[1], split, seq_order=order)
        for layer in range(layers):
            p = layer % pools
            i = layer % nq
            kp, vp = backend.k_cache[p], backend.v_cache[p]
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            # the step's new token written by the decode launch itself (one launch per layer)
            ops.paged_decode_append(q[i], k_new[i], v_new[i], slots, kp, vp, tables, ctx, scale,
                                    split, out=out[i], workspace=ws, device_error=err,
                                    seq_order=order, planned=bool(split))
            if record:
                e1.record(stream)
                dec_events.append((e0, e1))

    ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
    dec_ms = sum(a.elapsed_time(z) for a, z in dec_events) / max(1, len(dec_events))
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")

    # ---- verification against the oracle (not timed): a sample on the CPU (the
    # oracle as pinned to the reference's fixtures) and every sequence of layer 0
    # with the oracle's steps run on the GPU in fp32.
    from oracle import oracle_decode

    sample = [0, b // 2, b - 1]
    layer0 = 0
    kp0, vp0 = backend.k_cache[0], backend.v_cache[0]
    ops.cache_append(kp0, vp0, k_new[layer0], v_new[layer0], slots, err)
    got = ops.paged_decode(q[layer0], kp0, vp0, tables, ctx, scale, split, workspace=ws)
    ref = oracle_decode(q[layer0][sample], kp0, vp0, wl.block_tables[sample],
                        wl.ctx_lens[sample])
    diff = (got[sample].float().cpu() - ref).abs()
    ok = bool((diff <= 2e-3 + 1e-2 * ref.abs()).all())
    ok_full, worst_full = verify_decode_full_batch(q[layer0], kp0, vp0, tables,
                                                   wl.ctx_lens.tolist(), got)
    verified, verified_full = ok, ok_full
    if world > 1:
        # NCCL over NVLink only for verification: gather every rank's flags and checksum.
        flags = [torch.zeros(3, dtype=torch.float64, device=dev) for _ in range(world)]
        mine = torch.tensor([1.0 if ok else 0.0, 1.0 if ok_full else 0.0,
                             float(got.float().sum())], dtype=torch.float64, device=dev)
        dist.all_gather(flags, mine)
        verified = all(bool(f[0].item()) for f in flags)
        verified_full = all(bool(f[1].item()) for f in flags)
        print(f"rank {rank}/{world}: verification all_gather over NCCL done "
              f"(flags {[tuple(int(x) for x in f[:2].tolist()) for f in flags]})",
              file=sys.stderr, flush=True)

    use_graph = not args.skip_graph and pools == layers
    if world > 1:  # every rank must take the same path (and the same collectives)
        flag = torch.tensor([1 if use_graph else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        use_graph = bool(flag.item())
    eager_ms = max_over_ranks(ms, world)
    total_seqs = sum_over_ranks(b, world)

    # ---- the step replayed from one CUDA graph (DecodeGraph): the headline when available
    graph_ms = layer_ms = own_graph_ms = clocks_g = None
    graph_same = None
    if use_graph:
        from paged_serve_b200.graphs import DecodeGraph

        dg = DecodeGraph(backend, batch=b, layers=layers, timing=True)
        for layer in range(layers):
            i = layer % nq
            dg.query[layer, :, 0].copy_(q[i])
            dg.key[layer, :, 0].copy_(k_new[i])
            dg.value[layer, :, 0].copy_(v_new[i])
        dg.load(wl.block_tables, wl.ctx_lens)
        graph_ms, clocks_g = timed_region(lambda record: dg.replay(), args.steps, args.warmup,
                                          world, local_rank)
        layer_ms = dg.layer_ms()  # every layer of the last timed replay
        eager0 = ops.paged_decode(q[0], backend.k_cache[0], backend.v_cache[0], tables, ctx,
                                  scale, split, workspace=ws)
        graph_same = bool(torch.equal(dg.outputs[0][:, 0], eager0))
        own_graph_ms = graph_ms
        graph_ms = max_over_ranks(graph_ms, world)
        del dg

    # ---- end to end through the public API, host buffers, copies inside the timed region
    e2e = None
    if not args.skip_e2e:
        pin = {"pin_memory": True}
        main = torch.cuda.current_stream(dev)
        up = torch.cuda.Stream(dev)
        down = torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(layers)]
        ev_done = [torch.cuda.Event() for _ in range(layers)]
        h_out = torch.empty((layers, b, 1, hq, d), dtype=dtype, **pin)
        if use_graph:
            # One graph per step holds the per-layer uploads (upload stream), the
            # layers, and the per-layer downloads (download stream); the step's
            # tables and lengths go up through load_decode before each replay.
            h_q = torch.empty((layers, b, 1, hq, d), dtype=dtype, **pin).normal_(0, 0.5)
            h_k = torch.empty((layers, b, 1, hkv, d), dtype=dtype, **pin).normal_(0, 0.5)
            h_v = torch.empty((layers, b, 1, hkv, d), dtype=dtype, **pin).normal_(0, 0.5)
            d_q = torch.empty((layers, b, 1, hq, d), dtype=dtype, device=dev)
            d_k = torch.empty((layers, b, 1, hkv, d), dtype=dtype, device=dev)
            d_v = torch.empty((layers, b, 1, hkv, d), dtype=dtype, device=dev)
            md_e = backend.static_decode_metadata(b)
            h_tables = wl.block_tables.clone()
            h_ctx = wl.ctx_lens.clone()

            def body():
                cap = torch.cuda.current_stream(dev)
                up.wait_stream(cap)
                down.wait_stream(cap)
                with torch.cuda.stream(up):
                    for layer in range(layers):
                        d_q[layer].copy_(h_q[layer], non_blocking=True)
                        d_k[layer].copy_(h_k[layer], non_blocking=True)
                        d_v[layer].copy_(h_v[layer], non_blocking=True)
                        ev_in[layer].record(up)
                for layer in range(layers):
                    cap.wait_event(ev_in[layer])
                    o = backend.forward(layer, d_q[layer], d_k[layer], d_v[layer], md_e)
                    ev_done[layer].record(cap)
                    down.wait_event(ev_done[layer])
                    with torch.cuda.stream(down):
                        h_out[layer].copy_(o, non_blocking=True)
                cap.wait_stream(up)
                cap.wait_stream(down)

            side = torch.cuda.Stream(dev)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                body()
            main.wait_stream(side)
            g_e2e = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_e2e):
                body()

            def e2e_step(record: bool):
                backend.load_decode(md_e, h_tables, h_ctx)
                g_e2e.replay()

            meta_h2d = md_e.block_tables.numel() * 4 + 4 * b * 4
            path = ("PagedCudaBackend static decode metadata (load_decode: tables and lengths "
                    "from host, one pinned upload + the device slot builder) + one CUDA graph "
                    "per step holding, per layer, the q/k/v upload, append + paged decode, and "
                    "the output download, uploads and downloads on their own streams")
        else:
            key_len = int(wl.ctx_lens.max())
            h_q = torch.empty((nq, b, 1, hq, d), dtype=dtype, **pin).normal_(0, 0.5)
            h_k = torch.empty((nq, b, 1, hkv, d), dtype=dtype, **pin).normal_(0, 0.5)
            h_v = torch.empty((nq, b, 1, hkv, d), dtype=dtype, **pin).normal_(0, 0.5)
            h_tables = wl.block_tables.clone().pin_memory()
            h_slots = slots.cpu().pin_memory()
            h_seq = wl.ctx_lens.clone().pin_memory()
            h_mask = (torch.arange(key_len).view(1, -1) >= (key_len - wl.ctx_lens.view(-1, 1)))
            h_mask = h_mask.pin_memory()
            d_q = torch.empty((layers, b, 1, hq, d), dtype=dtype, device=dev)
            d_k = torch.empty((layers, b, 1, hkv, d), dtype=dtype, device=dev)
            d_v = torch.empty((layers, b, 1, hkv, d), dtype=dtype, device=dev)

            ev_copied = [torch.cuda.Event() for _ in range(layers)]

            def e2e_step(record: bool):
                step = StepInput(query_len=1, context_len=key_len - 1,
                                 seq_lens=h_seq.to(dev, non_blocking=True),
                                 padding_mask=h_mask.to(dev, non_blocking=True), is_prefill=False,
                                 block_tables=h_tables.to(dev, non_blocking=True),
                                 slot_mapping=h_slots.to(dev, non_blocking=True))
                md = backend.begin_step(step)
                up.wait_stream(main)  # the previous step no longer reads d_q/d_k/d_v
                with torch.cuda.stream(up):
                    for layer in range(layers):
                        i = layer % nq
                        d_q[layer].copy_(h_q[i], non_blocking=True)
                        d_k[layer].copy_(h_k[i], non_blocking=True)
                        d_v[layer].copy_(h_v[i], non_blocking=True)
                        ev_in[layer].record(up)
                for layer in range(layers):
                    main.wait_event(ev_in[layer])
                    if layer >= pools:  # the decode output buffer of this pool is reused:
                        main.wait_event(ev_copied[layer - pools])  # its last copy is done
                    o = backend.forward(layer % pools, d_q[layer], d_k[layer], d_v[layer], md)
                    ev_done[layer].record(main)
                    down.wait_event(ev_done[layer])
                    o.record_stream(down)
                    with torch.cuda.stream(down):
                        h_out[layer].copy_(o, non_blocking=True)
                    ev_copied[layer].record(down)
                main.wait_stream(down)

            meta_h2d = (h_tables.numel() * 4 + h_slots.numel() * 8 + h_seq.numel() * 4
                        + h_mask.numel())
            path = ("PagedCudaBackend.begin_step + forward x layers (append + paged decode); "
                    "inputs uploaded on one stream, outputs downloaded per layer on another, "
                    "both overlapping compute")

        e2e_ms, _ = timed_region(e2e_step, args.steps, args.warmup, world, local_rank)
        e2e_ms = max_over_ranks(e2e_ms, world)
        h2d = meta_h2d + layers * (b * hq * d + 2 * b * hkv * d) * elem
        d2h = layers * b * hq * d * elem
        e2e = {"value": total_seqs * args.steps / (e2e_ms / 1e3),
               "unit": "tokens/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": e2e_ms / args.steps, "path": path}

    dec_ms_max = max_over_ranks(dec_ms, world)
    own_step_ms = own_graph_ms if use_graph else ms
    own_clocks = clocks_g if use_graph else clocks
    per_rank = gather_objects({
        "rank": rank, "sequences": b, "ctx_tokens": wl.total_tokens,
        "step_ms": own_step_ms / args.steps, "decode_launch_ms": dec_ms,
        "sm_mhz": (own_clocks or {}).get("sm_mhz"),
        "clock_reasons": (own_clocks or {}).get("reasons"),
        "power_cap_fraction": (own_clocks or {}).get("power_cap_fraction")}, world)
    loads = [r["ctx_tokens"] for r in per_rank]
    pk = peaks()
    algo = wl.algorithmic_bytes_per_layer(elem)
    traffic = profile_traffic(f"paged_decode_{args.workload}")
    eager = {"value": total_seqs * args.steps / (eager_ms / 1e3), "unit": "tokens/s",
             "ms_per_step": eager_ms / args.steps, "clocks": clocks,
             "decode_launch_ms": dec_ms,
             "decode_achieved_gbs": algo / (dec_ms / 1e3) / 1e9,
             "path": "per-layer ops.paged_decode_append (the decode launch also writes the "
                     "step's new token) launched from Python, CUDA events around every launch"}
    if use_graph:
        step_ms = graph_ms
        # one layer of the graph = the append of 256 new tokens + the decode (+ combine)
        append_bytes = b * 2 * (2 * hkv * d * elem) + b * 8
        lay_ms = sum(layer_ms) / len(layer_ms)
        achieved = (algo + append_bytes) / (lay_ms / 1e3) / 1e9
        roof_kernel = ("one decode layer inside the replayed graph: ps_paged_decode_append "
                       f"(writes the {b} new tokens, then decodes"
                       + (", + split-K plan and combine" if split else "") +
                       "); timed by event nodes around each layer")
        roof_ms, roof_bytes = lay_ms, algo + append_bytes
        clocks_line = clocks_g
    else:
        step_ms = eager_ms
        achieved = algo / (dec_ms / 1e3) / 1e9
        roof_kernel = "ps_paged_decode (decode + split-K combine)"
        roof_ms, roof_bytes = dec_ms, algo
        clocks_line = clocks
    line = {
        "metric": METRIC,
        "value": total_seqs * args.steps / (step_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms / args.steps,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded: ctx ~ U[512,4096], K/V/q ~ 0.5*N(0,1), shuffled block ids)"
        if args.workload in ("llama8b", "qwen05b")
        else "synthetic (seeded lognormal lengths, sigma 1.0)",
        "config": {
            "workload": f"{args.workload} decode: {layers} layers, Hq {hq}, Hkv {hkv}, D {d}, "
                        f"block 16, " + (f"{b} sequences/GPU" if weak else
                                         f"{int(total_seqs)} sequences sharded over {world} "
                                         f"GPU(s) by greedy token balance"),
            "global_batch": int(total_seqs),
            "ctx_tokens_per_gpu": wl.total_tokens,
            "split_tokens": split,
            "distinct_layer_pools": pools,
            "step_path": ("paged_serve_b200.graphs.DecodeGraph replay (one decode launch per "
                          "layer, appending the new token, in one CUDA graph)" if use_graph
                          else "eager launches"),
            "l2": "inputs larger than L2 (each layer's KV >> 126 MB), no flush needed",
            "parallelism": f"sequence-sharded x{world} (LPT), no hot-path collective",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": roof_kernel,
            "achieved": achieved,
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"],
            "frac_of_8tbs_spec": achieved / 8000.0,
            "peak_source": f"{pk['source']} hbm_gbs" + (" (of measured)" if pk["source"] ==
                                                         "measured" else " (of fallback)"),
            "traffic": traffic,
            "algorithmic_bytes_per_launch": roof_bytes,
            "launch_ms": roof_ms,
            "decode_launch_ms_eager_max_over_ranks": dec_ms_max,
        },
        "per_rank": per_rank,
        "token_imbalance_max_over_mean": max(loads) / (sum(loads) / len(loads)),
        "e2e": e2e,
        "eager": eager,
        "graph_bit_exact_vs_eager": graph_same,
        # per layer: one decode launch that also appends the new token (+ the
        # split-K plan and combine); the eager path adds one launch-order kernel
        # per step (the graph's is computed at load)
        "gpu_launches": args.steps * (layers * (1 + (2 if split and wl.block_tables.shape[1] *
                                                      s.block_size > split else 0))
                                      + (0 if use_graph else 1)),
        "clocks": clocks_line,
        "verified_vs_oracle": verified,
        "verified_full_batch_gpu_fp32": verified_full,
        "verification": ("3 sequences of layer 0 against the oracle on the CPU; all "
                         f"{b} sequences of layer 0 (per rank) against the oracle's steps on "
                         f"the GPU in fp32, worst |err|/bound {worst_full:.3f} on rank {rank}"),
    }
    if args.read_ceiling:
        rc = args.read_ceiling
        line["roofline"]["read_ceiling_gbs"] = rc["gbs"]
        line["roofline"]["frac_of_read_ceiling"] = achieved / rc["gbs"]
        line["roofline"]["read_ceiling"] = rc
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_decode_sample(wl, seqs=min(32, b), reps=2)
        line["cpu_baseline"] = {"value": cpu["tokens_per_s"], "unit": "tokens/s",
                                "cores": cpu["cores"], "kind": "port", "sample": cpu["sample"],
                                "extrapolated": True,
                                "sample_fraction_of_step": cpu["sample_fraction"]}
    backend.free()
    return line


# ----------------------------------------------------------------------------- continuous
def bench_continuous(args, rank: int, world: int, local_rank: int) -> dict:
    """The llama8b decode step driven by the block manager (continuous batching).

    Same sequences, pool size, shuffled block ids and kernels as the llama8b
    decode line; every step additionally runs the host scheduler
    (``BlockManager.append_slots`` + ``schedule``) and ``begin_plan`` (one
    pinned upload of tables and lengths, the device slot builder) before the
    layers, all inside the timed region. The cached prompts are the pool's
    random contents, as in the static line.
    """
    from paged_serve_b200 import ops
    from paged_serve_b200.backend import PagedCudaBackend
    from paged_serve_b200.block_manager import BlockManager
    from paged_serve_b200.config import ModelConfig
    from paged_serve_b200.workloads import decode_workload

    dev = torch.device("cuda", local_rank)
    wl = decode_workload("llama8b", seed=args.seed, rank=rank, world=world, weak=True,
                         batch=args.batch)
    s = wl.spec
    layers = args.layers or s.num_layers
    b, hq, hkv, d, bs = wl.batch, s.num_q_heads, s.num_kv_heads, s.head_dim, s.block_size
    dtype = torch.bfloat16
    elem = 2
    per_layer_pool = 2 * wl.num_blocks * hkv * bs * d * elem
    free, _ = torch.cuda.mem_get_info(dev)
    pools = max(1, min(layers, (int(free * 0.80) - (256 << 20)) // per_layer_pool))
    grow = args.steps + args.warmup + 2
    max_len = int(wl.ctx_lens.max()) + grow
    model = ModelConfig(s.name, num_layers=pools, num_q_heads=hq, num_kv_heads=hkv, head_dim=d,
                        rope_theta=s.rope_theta)
    backend = PagedCudaBackend(model, device=dev, dtype=dtype, block_size=bs,
                               num_blocks=wl.num_blocks, split_tokens=args.split_tokens)
    backend.allocate(num_seq_slots=b, max_seq_len=max_len)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
    backend.k_cache.normal_(0.0, s.value_scale, generator=gen)
    backend.v_cache.normal_(0.0, s.value_scale, generator=gen)
    perm = torch.randperm(wl.num_blocks, generator=torch.Generator().manual_seed(args.seed))
    mgr = BlockManager(wl.num_blocks, bs, free_order=perm.tolist())
    ids = list(range(b))
    for i in ids:  # every prompt but its newest token is cached
        mgr.allocate(i, int(wl.ctx_lens[i]) - 1)
    mgr.schedule(ids)
    width = backend.max_blocks_per_seq

    nq = min(layers, 32)
    q = torch.empty((nq, b, hq, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    k_new = torch.empty((nq, b, hkv, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    out = torch.empty((nq, b, hq, d), dtype=dtype, device=dev)
    ws = backend._workspace
    err = backend.device_error
    scale = 1.0 / math.sqrt(d)
    split = args.split_tokens
    stream = torch.cuda.current_stream(dev)
    dec_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
    host_s: list[float] = []
    algo_steps: list[int] = []
    state = {}

    def run_step(record: bool):
        t0 = time.perf_counter()
        for i in ids:
            mgr.append_slots(i, 1)
        plan = mgr.schedule(ids)
        md = backend.begin_plan(plan, width=width)
        if record:
            host_s.append(time.perf_counter() - t0)
            lens = plan.seq_lens
            algo_steps.append(sum(lens) * 2 * hkv * d * elem + 2 * b * hq * d * elem
                              + sum(-(-n // bs) for n in lens) * 4)
        state["md"] = md
        for layer in range(layers):
            p = layer % pools
            i = layer % nq
            kp, vp = backend.k_cache[p], backend.v_cache[p]
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            ops.paged_decode_append(q[i], k_new[i], v_new[i], md.slot_mapping, kp, vp,
                                    md.block_tables, md.ctx_lens, scale, split, out=out[i],
                                    workspace=ws, device_error=err, seq_order=md.seq_order)
            if record:
                e1.record(stream)
                dec_events.append((e0, e1))

    ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
    dec_ms = sum(a.elapsed_time(z) for a, z in dec_events) / max(1, len(dec_events))
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")

    # verification of a sample against the oracle through the manager's own tables
    from oracle import oracle_decode

    md = state["md"]
    sample = [0, b // 2, b - 1]
    kp0, vp0 = backend.k_cache[0], backend.v_cache[0]
    got = ops.paged_decode(q[0], kp0, vp0, md.block_tables, md.ctx_lens, scale, split,
                           workspace=ws)
    ref = oracle_decode(q[0][sample], kp0, vp0, md.block_tables.cpu()[sample],
                        md.ctx_lens.cpu()[sample])
    diff = (got[sample].float().cpu() - ref).abs()
    verified = bool((diff <= 2e-3 + 1e-2 * ref.abs()).all())
    if world > 1:
        flags = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(flags, torch.tensor([1.0 if verified else 0.0], dtype=torch.float64,
                                            device=dev))
        verified = all(bool(f.item()) for f in flags)

    ms = max_over_ranks(ms, world)
    pk = peaks()
    algo = sum(algo_steps) / len(algo_steps)
    achieved = algo / (dec_ms / 1e3) / 1e9
    total_seqs = sum_over_ranks(b, world)
    line = {
        "metric": METRIC,
        "value": total_seqs * args.steps / (ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded: ctx ~ U[512,4096], K/V/q ~ 0.5*N(0,1), shuffled block ids)",
        "config": {
            "workload": f"llama8b decode, continuous batching: BlockManager.append_slots + "
                        f"schedule + PagedCudaBackend.begin_plan per step, then {layers} layers "
                        f"of append + paged decode; Hq {hq}, Hkv {hkv}, D {d}, block {bs}, "
                        f"{b} sequences/GPU",
            "global_batch": int(total_seqs),
            "split_tokens": split,
            "distinct_layer_pools": pools,
            "host_schedule_ms_per_step": 1e3 * sum(host_s) / len(host_s),
            "l2": "inputs larger than L2 (each layer's KV >> 126 MB), no flush needed",
            "parallelism": f"sequence-sharded x{world} (LPT), no hot-path collective",
        },
        "roofline": {
            "bound": "hbm", "kernel": "ps_paged_decode", "achieved": achieved,
            "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": profile_traffic("paged_decode_llama8b"),
            "algorithmic_bytes_per_launch": algo, "launch_ms": dec_ms,
        },
        # per step: slot builder + launch order, then one decode-with-append per layer
        "gpu_launches": args.steps * (2 + layers),
        "clocks": clocks,
        "verified_vs_oracle": verified,
    }
    backend.free()
    return line


# ----------------------------------------------------------------------------- mixed
def bench_mixed(args, rank: int, world: int, local_rank: int) -> dict:
    """Continuous batching with chunked prefill: every step, 255 sequences of the
    llama8b workload decode one token while one long prompt prefills its next
    64-token chunk, all 32 layers, through BlockManager.schedule +
    PagedCudaBackend.begin_plan + forward. The same steps are timed with the
    mixed-step split (one-token sequences through the decode kernel, the chunk
    through the prefill kernel) and without it (every sequence through the
    prefill kernel), alternating in one run.
    """
    from paged_serve_b200.backend import PagedCudaBackend
    from paged_serve_b200.block_manager import BlockManager
    from paged_serve_b200.config import ModelConfig
    from paged_serve_b200.workloads import decode_workload

    dev = torch.device("cuda", local_rank)
    wl = decode_workload("llama8b", seed=args.seed, rank=rank, world=world, weak=True,
                         batch=args.batch)
    s = wl.spec
    layers = args.layers or s.num_layers
    hq, hkv, d, bs = s.num_q_heads, s.num_kv_heads, s.head_dim, s.block_size
    chunk = 64
    dec = wl.batch - 1
    total_steps = 6 * (args.steps + args.warmup) + 4  # six timed regions + the check
    prompt_blocks = (chunk * total_steps + bs - 1) // bs
    num_blocks = wl.num_blocks + prompt_blocks + total_steps * dec // bs + 64
    per_layer_pool = 2 * num_blocks * hkv * bs * d * 2
    free, _ = torch.cuda.mem_get_info(dev)
    pools = max(1, min(layers, (int(free * 0.75) - (1 << 30)) // per_layer_pool))
    max_len = max(int(wl.ctx_lens.max()) + total_steps, chunk * total_steps)
    model = ModelConfig(s.name, num_layers=pools, num_q_heads=hq, num_kv_heads=hkv, head_dim=d,
                        rope_theta=s.rope_theta)
    backend = PagedCudaBackend(model, device=dev, dtype=torch.bfloat16, block_size=bs,
                               num_blocks=num_blocks, split_tokens=args.split_tokens)
    backend.allocate(num_seq_slots=wl.batch, max_seq_len=max_len)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
    backend.k_cache.normal_(0.0, s.value_scale, generator=gen)
    backend.v_cache.normal_(0.0, s.value_scale, generator=gen)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(args.seed))
    mgr = BlockManager(num_blocks, bs, free_order=perm.tolist())
    ids = list(range(wl.batch))
    for i in range(dec):  # every prompt but its newest token is cached
        mgr.allocate(i, int(wl.ctx_lens[i]) - 1)
    mgr.allocate(dec, chunk)  # the long prompt's first chunk
    mgr.schedule(ids[:dec])
    width = backend.max_blocks_per_seq
    q = torch.empty((wl.batch, chunk, hq, d), dtype=torch.bfloat16, device=dev).normal_(
        0, 0.5, generator=gen)
    k_new = torch.empty((wl.batch, chunk, hkv, d), dtype=torch.bfloat16, device=dev).normal_(
        0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    state = {"first": True}

    def run_step(record: bool):
        for i in range(dec):
            mgr.append_slots(i, 1)
        if not state["first"]:
            mgr.append_slots(dec, chunk)
        state["first"] = False
        plan = mgr.schedule(ids)
        md = backend.begin_plan(plan, width=width)
        for layer in range(layers):
            backend.forward(layer % pools, q, k_new, v_new, md)

    results = {}
    modes = ("overlap", "serial", "plain")  # split + side stream, split, no split
    for mode in modes + modes:
        backend.split_mixed_steps = mode != "plain"
        backend.overlap_mixed_steps = mode == "overlap"
        ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
        ms = max_over_ranks(ms, world)
        results.setdefault(mode, []).append((ms / args.steps, clocks))
    code = int(backend.device_error.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")
    # verification (not timed): one more mixed step, layer 0, a decoding sequence and
    # the prefilling one against the oracle through the manager's own tables
    from oracle import oracle_prefill

    for i in range(dec):
        mgr.append_slots(i, 1)
    mgr.append_slots(dec, chunk)
    plan = mgr.schedule(ids)
    backend.split_mixed_steps = backend.overlap_mixed_steps = True
    md = backend.begin_plan(plan, width=width)
    out = backend.forward(0, q, k_new, v_new, md)
    tq = plan.query_len
    flat_q = q.reshape(-1, hq, d)
    pick = [0, dec // 2, dec]
    ref = oracle_prefill(flat_q, backend.k_cache[0], backend.v_cache[0], md.block_tables.cpu(),
                         md.q_starts.cpu(), md.q_lens.cpu(), md.ctx_before.cpu(), seqs=pick)
    verified = True
    for i in pick:
        n = plan.q_lens[i]
        got = out[i, tq - n :].float().cpu()
        verified = verified and bool(((got - ref[i]).abs() <= 2e-3 + 1e-2 * ref[i].abs()).all())
    if world > 1:
        verified = all(gather_objects(verified, world))
    split_ms = min(m for m, _ in results["overlap"])
    serial_ms = min(m for m, _ in results["serial"])
    plain_ms = min(m for m, _ in results["plain"])
    toks = sum_over_ranks(dec + chunk, world)
    line = {
        "metric": "continuous batching with chunked prefill: tokens/s (decode + prefill)",
        "value": toks / (split_ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": split_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded: llama8b lengths, 0.5*N(0,1) K/V/q)",
        "config": {"workload": f"mixed: {dec} sequences decode 1 token + 1 prompt prefills a "
                               f"{chunk}-token chunk per step, {layers} layers, Hq {hq}, Hkv {hkv}, "
                               f"D {d}, block {bs}; steps laid out [B, {chunk}] left-padded",
                   "distinct_layer_pools": pools, "split_tokens": args.split_tokens},
        "split_mixed_ms_per_step": [m for m, _ in results["overlap"]],
        "split_serial_ms_per_step": [m for m, _ in results["serial"]],
        "prefill_kernel_for_all_ms_per_step": [m for m, _ in results["plain"]],
        "speedup_of_split": plain_ms / split_ms,
        "speedup_of_overlap": serial_ms / split_ms,
        "step_path": "split mixed step: append, then the chunk's prefill on the current stream "
                     "beside the one-token sequences' listed decode on a side stream",
        "clocks": results["overlap"][-1][1],
        "verified_vs_oracle": verified,
        "verification": f"sequences {pick} of layer 0 (decoding and prefilling) against the "
                        "oracle on the CPU",
        "gpu_launches": args.steps * (2 + 3 * layers),
    }
    backend.free()
    return line


# ----------------------------------------------------------------------------- swap
def bench_swap(args, rank: int, world: int, local_rank: int) -> dict:
    """Swap-out + swap-in of 512 llama8b blocks (all 32 layers, K and V: 1 GiB each way).

    HBM side: shuffled block ids of a 4096-block pool; host side: consecutive
    blocks of a pinned pool, as a fresh host free list hands them out. Each step
    moves the blocks out and back in (to other HBM blocks) with two
    ``ps_swap_blocks`` launches. The denominator is the copy engine's bandwidth
    for one contiguous 1 GiB transfer each way, measured in the same run.
    """
    from paged_serve_b200 import ops

    dev = torch.device("cuda", local_rank)
    layers, hkv, bs, d = 32, 8, 16, 128
    nb, nh, npairs = 4096, 512, 512
    dtype = torch.bfloat16
    shape = (layers, nb, hkv, bs, d)
    k = torch.empty(shape, dtype=dtype, device=dev).normal_()
    v = torch.empty(shape, dtype=dtype, device=dev).normal_()
    hk = torch.empty((layers, nh, hkv, bs, d), dtype=dtype, pin_memory=True)
    hv = torch.empty_like(hk, pin_memory=True)
    g = torch.Generator().manual_seed(args.seed + rank)
    perm = torch.randperm(nb, generator=g)
    out_pairs = torch.stack([perm[:npairs], torch.arange(npairs)], 1).contiguous().to(dev)
    in_pairs = torch.stack([torch.arange(npairs), perm[npairs : 2 * npairs]], 1).contiguous()
    in_pairs = in_pairs.to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    block_bytes = hkv * bs * d * 2
    moved = npairs * layers * 2 * block_bytes  # bytes per direction
    stream = torch.cuda.current_stream(dev)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(reps):
            a, z = ev(), ev()
            a.record(stream)
            fn()
            z.record(stream)
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(z))
        return best

    # copy-engine reference: one contiguous transfer of the same byte count
    flat_d = torch.empty(moved // 2, dtype=dtype, device=dev)
    flat_h = torch.empty(moved // 2, dtype=dtype, pin_memory=True)
    ce_d2h = moved / (timed(lambda: flat_h.copy_(flat_d, non_blocking=True)) / 1e3) / 1e9
    ce_h2d = moved / (timed(lambda: flat_d.copy_(flat_h, non_blocking=True)) / 1e3) / 1e9
    del flat_d, flat_h

    sweep = {}
    for cap in (16, 32, 64, 148, 296, 592):
        t_out = timed(lambda: ops.swap_blocks(hk, hv, k, v, out_pairs, cap, err))
        t_in = timed(lambda: ops.swap_blocks(k, v, hk, hv, in_pairs, cap, err))
        sweep[cap] = {"out_gbs": moved / (t_out / 1e3) / 1e9, "in_gbs": moved / (t_in / 1e3) / 1e9}
    cap = 0  # the library default (32 CTAs for host-side moves) in the timed region

    events = []

    def run_step(record: bool):
        a, m, z = ev(), ev(), ev()
        a.record(stream)
        ops.swap_blocks(hk, hv, k, v, out_pairs, cap, err)
        m.record(stream)
        ops.swap_blocks(k, v, hk, hv, in_pairs, cap, err)
        z.record(stream)
        if record:
            events.append((a, m, z))

    ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
    t_out = sum(a.elapsed_time(m) for a, m, _ in events) / len(events)
    t_in = sum(m.elapsed_time(z) for _, m, z in events) / len(events)
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")
    # bit-exact check of the last round trip (not timed)
    sample = torch.arange(0, npairs, 37)
    ok = torch.equal(hk[:, sample], k[:, perm[sample]].cpu()) and torch.equal(
        k[:, perm[npairs + sample]].cpu(), hk[:, sample])

    # conventional baseline: one cudaMemcpyAsync per (pair, layer, K|V), 64 pairs only
    sub = 64
    src_ids, dst_ids = perm[:sub].tolist(), list(range(sub))

    def per_block():
        for layer in range(layers):
            for sblk, hblk in zip(src_ids, dst_ids, strict=True):
                hk[layer, hblk].copy_(k[layer, sblk], non_blocking=True)
                hv[layer, hblk].copy_(v[layer, sblk], non_blocking=True)

    t0 = time.perf_counter()
    per_block()
    torch.cuda.synchronize()
    pb_gbs = sub * layers * 2 * block_bytes / (time.perf_counter() - t0) / 1e9

    ms = max_over_ranks(ms, world)
    out_gbs = moved / (t_out / 1e3) / 1e9
    in_gbs = moved / (t_in / 1e3) / 1e9
    total = sum_over_ranks(2 * moved, world)
    return {
        "metric": "KV swap-out + swap-in GB/s (pinned host <-> HBM blocks)",
        "value": total * args.steps / (ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) pool, shuffled HBM block ids)",
        "config": {"workload": f"swap: {npairs} blocks x {layers} layers x K,V of "
                               f"{block_bytes // 1024} KB = {moved >> 20} MiB each way; "
                               f"HBM pool {nb} blocks, host pool {nh} blocks (pinned)",
                   "max_ctas": "library default (32 CTAs when one side is host memory)",
                   "ctas_sweep": sweep,
                   "l2": "1 GiB per direction, larger than L2"},
        "roofline": {"bound": "host link", "kernel": "ps_swap_blocks",
                     "achieved": {"out": out_gbs, "in": in_gbs},
                     "peak": {"out": ce_d2h, "in": ce_h2d}, "unit": "GB/s",
                     "frac": {"out": out_gbs / ce_d2h, "in": in_gbs / ce_h2d},
                     "peak_source": "copy engine, one contiguous 1 GiB transfer each way, "
                                    "measured in this run",
                     "traffic": None, "algorithmic_bytes_per_launch": moved},
        "per_block_memcpy_gbs": pb_gbs,
        "per_block_memcpy": f"one cudaMemcpyAsync per (block, layer, K|V): {sub} blocks, "
                            f"{sub * layers * 2} copies, host-timed",
        "gpu_launches": 2 * args.steps, "clocks": clocks, "verified_bit_exact": bool(ok),
    }


# ----------------------------------------------------------------------------- append
def bench_append(args, rank: int, world: int, local_rank: int) -> dict:
    from paged_serve_b200 import ops
    from paged_serve_b200.rope import cos_sin_table
    from paged_serve_b200.workloads import append_workload

    dev = torch.device("cuda", local_rank)
    wl = append_workload(seed=args.seed + rank)
    layers = args.layers or wl.num_layers
    dtype = torch.bfloat16
    shape = (layers, wl.num_blocks, wl.num_kv_heads, wl.block_size, wl.head_dim)
    k_pool = torch.zeros(shape, dtype=dtype, device=dev)
    v_pool = torch.zeros_like(k_pool)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    kshape = (layers, wl.num_tokens, wl.num_kv_heads, wl.head_dim)
    key = torch.empty(kshape, dtype=dtype, device=dev).normal_(generator=gen)
    value = torch.empty(kshape, dtype=dtype, device=dev).normal_(generator=gen)
    slots = wl.slot_mapping.to(dev)
    pos = wl.positions.to(dev)
    table = cos_sin_table(wl.head_dim, wl.rope_theta, 4096, dtype, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    events = []

    def run_step(record):
        for layer in range(layers):
            if record:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            ops.cache_append_rope(k_pool[layer], v_pool[layer], key[layer], value[layer], slots,
                                  pos, table, err)
            if record:
                e1.record(stream)
                events.append((e0, e1))

    ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
    launch_ms = sum(a.elapsed_time(z) for a, z in events) / len(events)
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")
    graph = None
    if not args.skip_graph:
        # the same 32 launches captured once and replayed per step
        eager_k = k_pool.clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            run_step(False)
        stream.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_step(False)
        g_ms, g_clocks = timed_region(lambda record: g.replay(), args.steps, args.warmup, world,
                                      local_rank)
        torch.cuda.synchronize()
        g_ms = max_over_ranks(g_ms, world)
        graph = {"value": sum_over_ranks(wl.num_tokens * layers, world) * args.steps
                 / (g_ms / 1e3), "unit": "token-layers/s", "ms_per_step": g_ms / args.steps,
                 "bit_exact_vs_eager": bool(torch.equal(k_pool, eager_k)), "clocks": g_clocks,
                 "path": "the 32 per-layer ps_cache_append_rope launches captured in one CUDA "
                         "graph, replayed per step"}
    # bit-exact check of the last layer's written rows against the oracle (not timed)
    from oracle import oracle_append

    last = layers - 1
    t = wl.num_tokens
    rows_k = torch.zeros((t, wl.num_kv_heads, 1, wl.head_dim), dtype=dtype)
    exp_k, exp_v = oracle_append(rows_k, rows_k.clone(), key[last], value[last],
                                 torch.arange(t), wl.positions, table)
    blk, off = slots // wl.block_size, slots % wl.block_size
    verified = bool(torch.equal(k_pool[last][blk, :, off, :].cpu(), exp_k[:, :, 0]) and
                    torch.equal(v_pool[last][blk, :, off, :].cpu(), exp_v[:, :, 0]))
    if world > 1:
        flags = gather_objects(verified, world)
        verified = all(flags)
    ms = max_over_ranks(ms, world)
    pk = peaks()
    algo = wl.algorithmic_bytes_per_layer(2)
    tokens = sum_over_ranks(wl.num_tokens * layers, world)
    eager = {"value": tokens * args.steps / (ms / 1e3), "unit": "token-layers/s",
             "ms_per_step": ms / args.steps, "launch_ms_events": launch_ms,
             "achieved_gbs_events": algo / (launch_ms / 1e3) / 1e9, "clocks": clocks,
             "path": "32 launches from Python with CUDA events around each"}
    if graph is not None:
        step_ms = graph["ms_per_step"] * args.steps
        # average launch = the graph's step time over its 32 back-to-back launches
        # (gaps between the launches included)
        per_launch = graph["ms_per_step"] / layers
        kernel = ("ps_cache_append_rope, 32 back-to-back launches in one replayed CUDA graph; "
                  "launch_ms = step time / 32 (inter-launch gaps included)")
        clocks_line = graph["clocks"]
    else:
        step_ms, per_launch = ms, launch_ms
        kernel = "ps_cache_append_rope (CUDA events around each launch)"
        clocks_line = clocks
    achieved = algo / (per_launch / 1e3) / 1e9
    return {
        "metric": "KV append + fused RoPE tokens/s (x layers)", "value":
        tokens * args.steps / (step_ms / 1e3), "unit": "token-layers/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": {"workload": f"append: {wl.num_tokens} tokens x {layers} layers, Hkv 8, D 128",
                   "step_path": "CUDA graph replay" if graph is not None else "eager launches",
                   "l2": "68 MB K/V per layer in, scattered over a 3 GB pool"},
        "roofline": {"bound": "hbm", "kernel": kernel, "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "traffic": profile_traffic("cache_append_rope_append"),
                     "algorithmic_bytes_per_launch": algo, "launch_ms": per_launch},
        "gpu_launches": args.steps * layers, "clocks": clocks_line, "eager": eager,
        "graph_bit_exact_vs_eager": None if graph is None else graph["bit_exact_vs_eager"],
        "verified_bit_exact_vs_oracle": verified,
        "verification": f"all {wl.num_tokens} rows of the last layer (K rotated, V) against "
                        "the oracle's reference RoPE + index_put, bit for bit",
        "cpu_baseline": cpu_append_sample(wl) if rank == 0 and world == 1 and not args.skip_cpu
        else None,
    }


# ----------------------------------------------------------------------------- long prompt
def bench_longprompt(args, rank: int, world: int, local_rank: int) -> dict:
    """One long prompt's next chunk: 512 new tokens attending the 32,256 tokens of
    the same prompt already cached (32,768 in all), Llama-3-8B attention geometry
    (Hq 32, Hkv 8, D 128, block 16), one layer; each step appends the chunk's K/V
    and prefills it. Its 64 work items (query-tile pairs x KV heads) would fill
    under half of the SMs, each walking 256 key tiles; split-K cuts every item's
    key range into pieces (the backend's policy, ops.prefill_split_keys) and a
    second launch merges them. Timed split and whole, alternating.
    """
    from paged_serve_b200 import ops

    dev = torch.device("cuda", local_rank)
    hq, hkv, d, bs = 32, 8, 128, 16
    chunk, total = 512, 32768
    ctx = total - chunk
    nblk = total // bs
    num_blocks = nblk + 64
    dtype = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
    shape = (num_blocks, hkv, bs, d)
    k_pool = torch.empty(shape, dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    v_pool = torch.empty(shape, dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(args.seed + rank))
    blocks = perm[:nblk]
    tables = blocks.to(torch.int32).view(1, nblk).to(dev)
    q = torch.empty((chunk, hq, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    k_new = torch.empty((chunk, hkv, d), dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    pos = torch.arange(ctx, total)
    slots = (blocks[pos // bs] * bs + pos % bs).to(torch.int64).to(dev)
    q_starts = torch.zeros(1, dtype=torch.int32, device=dev)
    q_lens = torch.tensor([chunk], dtype=torch.int32, device=dev)
    ctx_lens = torch.tensor([ctx], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(d)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    items = hkv * -(-chunk // (2 * (128 // (hq // hkv))))
    split = ops.prefill_split_keys(items, total, sms)
    ws = torch.empty(max(ops.prefill_workspace_bytes(1, chunk, hq, hkv, d, bs, nblk, split), 256),
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    steps = max(args.steps, 50)

    def prefill(keys: int) -> None:
        ops.paged_prefill(q, k_pool, v_pool, tables, q_starts, q_lens, ctx_lens, chunk, scale,
                          out=out, device_error=err, split_keys=keys,
                          workspace=ws if keys else None)

    def step_fn(keys: int):
        def run_step(record: bool) -> None:
            ops.cache_append(k_pool, v_pool, k_new, v_new, slots, err)
            prefill(keys)
        return run_step

    results = {}
    for mode in ("split", "whole", "split", "whole"):
        ms, clocks = timed_region(step_fn(split if mode == "split" else 0), steps, args.warmup,
                                  world, local_rank)
        results.setdefault(mode, []).append((max_over_ranks(ms, world) / steps, clocks))
    # the prefill call alone (both launches when split), back to back, after 1 s idle
    launch = {}
    for mode, keys in (("split", split), ("whole", 0)):
        torch.cuda.synchronize()
        time.sleep(1.0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(20):
            prefill(keys)
        e1.record(stream)
        torch.cuda.synchronize()
        launch[mode] = max_over_ranks(e0.elapsed_time(e1) / 20, world)
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")
    # verification (not timed): the split output against the oracle's steps on
    # the GPU in fp32 for every row, and against the whole-item kernel
    from oracle import oracle_prefill

    prefill(split)
    got = out.float().clone()
    prefill(0)
    whole = out.float().clone()
    ref = oracle_prefill(q, k_pool, v_pool, tables.cpu(), q_starts.cpu(), q_lens.cpu(),
                         ctx_lens.cpu(), device=dev)[0].to(dev)
    worst = float(((got - ref).abs() / (2e-3 + 1e-2 * ref.abs())).max())
    worst_whole = float(((got - whole).abs() / (2e-3 + 1e-2 * whole.abs())).max())
    verified = worst <= 1.0 and worst_whole <= 1.0
    if world > 1:
        verified = all(gather_objects(verified, world))
    split_ms = min(m for m, _ in results["split"])
    whole_ms = min(m for m, _ in results["whole"])
    pk = peaks()
    flops = 4 * d * hq * (chunk * ctx + chunk * (chunk + 1) // 2)
    achieved = flops / (launch["split"] / 1e3) / 1e12
    line = {
        "metric": "long-prompt chunked prefill tokens/s", "unit": "tokens/s",
        "value": sum_over_ranks(chunk, world) / (split_ms / 1e3), "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": split_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded 0.5*N(0,1) K/V/q, shuffled block ids)",
        "config": {"workload": f"longprompt: one prompt's {chunk}-token chunk over its {ctx} "
                               f"cached tokens, Hq {hq}, Hkv {hkv}, D {d}, block {bs}, one layer",
                   "split_keys": split, "work_items": items,
                   "pieces_per_item": -(-total // split) if split else 1},
        "split_ms_per_step": [m for m, _ in results["split"]],
        "whole_ms_per_step": [m for m, _ in results["whole"]],
        "speedup_of_split": whole_ms / split_ms,
        "roofline": {"bound": "tensor", "kernel": "ps_paged_prefill_split (prefill + combine)",
                     "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["bf16_tflops"],
                     "peak_source": f"{pk['source']} bf16_tflops (burst)" + (
                         " (of measured)" if pk["source"] == "measured" else " (of fallback)"),
                     "traffic": profile_traffic("paged_prefill_split_longprompt"),
                     "algorithmic_flops_per_launch": flops,
                     "launch_ms": launch["split"], "launch_ms_whole": launch["whole"],
                     "how": "20 back-to-back calls after 1 s idle, CUDA events around the 20 "
                            "(max over ranks)"},
        "gpu_launches": steps * (3 if split else 2), "clocks": results["split"][-1][1],
        "step": "ps_cache_append (the chunk's K/V) + ps_paged_prefill_split",
        "verified_vs_oracle": verified,
        "verification": f"all {chunk} rows against the oracle's steps on the GPU in fp32 (worst "
                        f"|err|/bound {worst:.3f}) and against the whole-item kernel "
                        f"({worst_whole:.3f})",
        "cpu_baseline": cpu_longprompt_sample(q, k_pool, v_pool, blocks, ctx, bs)
        if rank == 0 and world == 1 and not args.skip_cpu else None,
    }
    return line


def cpu_longprompt_sample(q, k_pool, v_pool, blocks, ctx: int, bs: int, rows: int = 32) -> dict:
    """The reference's contiguous prefill (the oracle, fp32) on the CPU for the first
    ``rows`` tokens of the chunk, each over the whole cached prompt; the chunk's
    other tokens attend as many keys (to within 1.6%), so tokens/s carries over."""
    from oracle import contiguous_attention

    n = ctx + rows
    ids = blocks[: -(-n // bs)].long()
    kk = k_pool.cpu()[ids].permute(0, 2, 1, 3).reshape(-1, k_pool.shape[1], k_pool.shape[3])[:n]
    vv = v_pool.cpu()[ids].permute(0, 2, 1, 3).reshape(-1, v_pool.shape[1], v_pool.shape[3])[:n]
    qq = q.cpu()[:rows].float()[None]
    mask = torch.ones((1, n), dtype=torch.bool)
    args = (qq, kk.float()[None], vv.float()[None], mask, ctx)
    contiguous_attention(*args)
    t0 = time.perf_counter()
    contiguous_attention(*args)
    sec = time.perf_counter() - t0
    return {"value": rows / sec, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"the chunk's first {rows} tokens over {ctx} cached + themselves "
                      "(fp32 contiguous attention)"}


# ----------------------------------------------------------------------------- prefix prefill
def bench_prefix(args, rank: int, world: int, local_rank: int) -> dict:
    from paged_serve_b200 import ops
    from paged_serve_b200.workloads import prefix_workload

    dev = torch.device("cuda", local_rank)
    wl = prefix_workload(seed=args.seed + rank)
    dtype = torch.bfloat16
    shape = (wl.num_blocks, wl.num_kv_heads, wl.block_size, wl.head_dim)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    k_pool = torch.empty(shape, dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    v_pool = torch.empty(shape, dtype=dtype, device=dev).normal_(0, 0.5, generator=gen)
    t = wl.total_q
    q = torch.empty((t, wl.num_q_heads, wl.head_dim), dtype=dtype, device=dev).normal_(
        0, 0.5, generator=gen)
    k_new = torch.empty((t, wl.num_kv_heads, wl.head_dim), dtype=dtype, device=dev).normal_(
        0, 0.5, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, 0.5, generator=gen)
    out = torch.empty_like(q)
    tables = wl.block_tables.to(dev)
    pairs = wl.cow_pairs.to(dev)
    slots = wl.slot_mapping.to(dev)
    q_starts, q_lens, ctx = wl.q_starts.to(dev), wl.q_lens.to(dev), wl.prefix_lens.to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(wl.head_dim)
    stream = torch.cuda.current_stream(dev)
    mq = int(wl.q_lens.max())

    def prefill():
        ops.paged_prefill(q, k_pool, v_pool, tables, q_starts, q_lens, ctx, mq, scale, out=out,
                          device_error=err)

    def run_step(record):
        ops.copy_blocks(k_pool, v_pool, pairs, err)
        ops.cache_append(k_pool, v_pool, k_new, v_new, slots, err)
        prefill()

    # the step (copy-on-write copy, suffix append, prefill): value and ms_per_step
    ms, clocks = timed_region(run_step, args.steps, args.warmup, world, local_rank)
    # the kernel's own launch time (the roofline): the same number of prefill
    # launches back to back, CUDA events around the region
    k_ms, k_clocks = timed_region(lambda record: prefill(), args.steps, args.warmup, world,
                                  local_rank)
    launch_ms = k_ms / args.steps
    # the prefill inside the step, with events around each launch (context only:
    # it starts behind the append's L2 write-backs, and the events keep the
    # next launch from starting early)
    in_step = []
    for _ in range(20):
        ops.copy_blocks(k_pool, v_pool, pairs, err)
        ops.cache_append(k_pool, v_pool, k_new, v_new, slots, err)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        prefill()
        e1.record(stream)
        in_step.append((e0, e1))
    torch.cuda.synchronize()
    in_step_ms = sum(a.elapsed_time(z) for a, z in in_step) / len(in_step)
    code = int(err.item())
    if code:
        raise RuntimeError(f"device error bits 0x{code:x} during the timed region")
    # verification (not timed): three sequences (one forked with copy-on-write)
    # against the oracle on the CPU, and every sequence with the oracle's steps
    # on the GPU in fp32
    from oracle import oracle_prefill

    args_o = (q, k_pool, v_pool, wl.block_tables, wl.q_starts, wl.q_lens, wl.prefix_lens)
    pick = [0, wl.batch // 2, wl.batch - 1]
    ref_cpu = oracle_prefill(*args_o, seqs=pick)
    ref_gpu = oracle_prefill(*args_o, device=dev)
    ok_cpu, worst = True, 0.0
    for i in range(wl.batch):
        r0 = int(wl.q_starts[i])
        got = out[r0 : r0 + int(wl.q_lens[i])].float()
        for ref, where in ((ref_gpu.get(i), "gpu"), (ref_cpu.get(i), "cpu")):
            if ref is None:
                continue
            ref = ref.to(dev)
            ratio = float(((got - ref).abs() / (2e-3 + 1e-2 * ref.abs())).max())
            if where == "cpu":
                ok_cpu = ok_cpu and ratio <= 1.0
            else:
                worst = max(worst, ratio)
    verified, verified_full = ok_cpu, worst <= 1.0
    if world > 1:
        flags = gather_objects((verified, verified_full), world)
        verified = all(f[0] for f in flags)
        verified_full = all(f[1] for f in flags)
    # burst: after a second idle, 20 back-to-back launches (~13 ms), before the
    # power controller reacts; the timed region above is long enough for it to
    # (the clock record shows sw_power_cap), so that one is the sustained figure
    torch.cuda.synchronize()
    time.sleep(1.0)
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    for _ in range(20):
        prefill()
    b1.record(stream)
    torch.cuda.synchronize()
    burst_ms = max_over_ranks(b0.elapsed_time(b1) / 20, world)
    ms = max_over_ranks(ms, world)
    launch_ms = max_over_ranks(launch_ms, world)
    in_step_ms = max_over_ranks(in_step_ms, world)
    pk = peaks()
    flops = wl.causal_flops()
    achieved = flops / (launch_ms / 1e3) / 1e12
    capped = bool(k_clocks and "sw_power_cap" in k_clocks.get("reasons", []))
    peak = pk["bf16_tflops_sustained"] if capped else pk["bf16_tflops"]
    peak_src = (f"{pk['source']} bf16_tflops_sustained (the timed region ran under the power "
                "cap: sw_power_cap in its clock record)" if capped else
                f"{pk['source']} bf16_tflops (burst)") + (
        " (of measured)" if pk["source"] == "measured" else " (of fallback)")
    burst = flops / (burst_ms / 1e3) / 1e12
    toks = sum_over_ranks(t, world)
    return {
        "metric": "prefix-cached paged prefill tokens/s", "value": toks * args.steps / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "prefix: 64 seqs x 512 new tokens over a shared 1024-token prefix "
                               "(8 fork at 1000 with CoW), Hq 32, Hkv 8, D 128, one layer"},
        "roofline": {"bound": "tensor", "kernel": "ps_paged_prefill", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": peak_src,
                     "traffic": profile_traffic("paged_prefill_prefix"),
                     "algorithmic_flops_per_launch": flops, "launch_ms": launch_ms,
                     "how": f"{args.steps} prefill launches back to back, CUDA events around "
                            "the region (max over ranks); clocks of that region",
                     "clocks": k_clocks,
                     "launch_ms_in_step": in_step_ms,
                     "frac_in_step": flops / (in_step_ms / 1e3) / 1e12 / peak},
        "roofline_burst": {"achieved": burst, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                           "frac": burst / pk["bf16_tflops"], "launch_ms": burst_ms,
                           "how": "20 back-to-back launches after 1 s idle, CUDA events around "
                                  "the 20 (max over ranks), against the burst peak"},
        "gpu_launches": args.steps * 3, "clocks": clocks,
        "step": "ps_copy_blocks (copy-on-write) + ps_cache_append (suffix K/V) + ps_paged_prefill",
        "verified_vs_oracle": verified,
        "verified_full_batch_gpu_fp32": verified_full,
        "verification": f"sequences {pick} (the last forks with copy-on-write) against the "
                        f"oracle on the CPU; all {wl.batch} with the oracle's steps on the GPU "
                        f"in fp32, worst |err|/bound {worst:.3f}",
        "cpu_baseline": cpu_prefix_sample(wl, k_pool, v_pool, q)
        if rank == 0 and world == 1 and not args.skip_cpu else None,
    }


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int) -> dict | None:
    """The reference's algorithm on the host CPU cores (rank 0 only)."""
    if rank != 0:
        return None
    from paged_serve_b200.workloads import decode_workload

    torch.set_num_threads(os.cpu_count() or 1)
    if args.workload not in ("llama8b", "llama70b"):
        return {"impl": "reference", "unavailable": f"no CPU reference arm for {args.workload}"}
    wl = decode_workload(args.workload, seed=args.seed, rank=0, world=1, weak=True,
                         batch=args.batch)
    s = wl.spec
    seqs = min(16, wl.batch)
    for _ in range(args.warmup):
        cpu_decode_sample(wl, seqs=seqs, reps=1)
    runs = [cpu_decode_sample(wl, seqs=seqs, reps=1) for _ in range(args.steps)]
    per = sum(r["seconds_per_sample"] for r in runs) / len(runs)
    value = statistics.median(r["tokens_per_s"] for r in runs)
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        # a step here is a bounded sample of the full decode step; ms_per_step is
        # the full step extrapolated from it (value = batch / that), and the time
        # actually spent per sample is sample_ms_per_step
        "ms_per_step": per * 1e3 / runs[0]["sample_fraction"],
        "sample_ms_per_step": per * 1e3,
        "extrapolated": True,
        "sample_fraction_of_step": runs[0]["sample_fraction"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": f"{args.workload} decode: {s.num_layers} layers, Hq "
                               f"{s.num_q_heads}, Hkv {s.num_kv_heads}, D {s.head_dim}, block 16,"
                               f" {wl.batch} sequences",
                   "global_batch": wl.batch},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": runs[0]["cores"],
                         "kind": "port", "sample": runs[0]["sample"], "extrapolated": True,
                         "sample_fraction_of_step": runs[0]["sample_fraction"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------- main
# Keys a sub-benchmark line keeps when it is attached to the headline line.
SUB_DROP = ("n_gpus", "higher_is_better", "vs_baseline", "data")


def sub_benchmarks(args, rank: int, world: int, local_rank: int) -> dict:
    """The other hot-path workloads, each with its own roofline, clocks,
    oracle check and CPU baseline, run after the headline on the same GPUs.

    ``append``: fused-RoPE append, 16640 tokens x 32 per-layer calls (one CUDA
    graph per step); ``prefill``: prefix-cached prefill with copy-on-write;
    ``llama70b``: the long-context skewed decode with one 512-sequence batch
    sharded over the ranks (strong scaling) and split-K over 512-token partitions;
    ``qwen05b``: decode at the reference's default model geometry (head dim 64,
    14 query heads over 2 KV heads) with the 8B workload's batch and lengths;
    ``mixed``: continuous batching with chunked prefill through the block manager
    (255 decodes + a 64-token prompt chunk per step), split vs prefill-only routing;
    ``longprompt``: a 512-token chunk of a 32k-token prompt, split-K vs whole items.
    """
    import copy
    import gc

    out = {}
    plan = (("append", bench_append, {"workload": "append", "steps": max(args.steps, 200)}),
            ("prefill", bench_prefix, {"workload": "prefix", "steps": max(args.steps, 200)}),
            ("llama70b", bench_decode, {"workload": "llama70b", "scaling": "strong",
                                        "split_tokens": 512, "skip_e2e": True,
                                        "batch": None, "layers": None}),
            ("qwen05b", bench_decode, {"workload": "qwen05b", "scaling": "weak",
                                       "split_tokens": 0, "skip_e2e": True,
                                       "batch": None, "layers": None}),
            ("mixed", bench_mixed, {"workload": "mixed", "split_tokens": 0, "batch": None,
                                    "layers": None}),
            ("longprompt", bench_longprompt, {"workload": "longprompt"}))
    for name, fn, over in plan:
        sub = copy.copy(args)
        for k, v in over.items():
            setattr(sub, k, v)
        gc.collect()
        torch.cuda.empty_cache()
        line = fn(sub, rank, world, local_rank)
        out[name] = {k: v for k, v in line.items() if k not in SUB_DROP}
    gc.collect()
    torch.cuda.empty_cache()
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-graph", action="store_true",
                    help="skip the CUDA-graph replay measurement")
    ap.add_argument("--workload",
                    choices=["llama8b", "llama70b", "qwen05b", "append", "prefix", "continuous",
                             "swap", "mixed", "longprompt"],
                    default="llama8b")
    ap.add_argument("--scaling", choices=["weak", "strong"], default=None,
                    help="weak: every rank draws its own batch (default for llama8b); strong: "
                         "one batch sharded over the ranks (default for llama70b)")
    ap.add_argument("--headline-only", action="store_true",
                    help="llama8b: skip the append / prefill / llama70b sub-results")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--split-tokens", type=int, default=None,
                    help="decode partition length (default 0 for llama8b, 512 for llama70b)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--batch", type=int, default=None, help="override sequences per GPU")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.split_tokens is None:
        args.split_tokens = 512 if args.workload == "llama70b" else 0
    if args.scaling is None:
        args.scaling = "strong" if args.workload == "llama70b" else "weak"
    args.read_ceiling = None

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload in ("llama8b", "llama70b", "qwen05b"):
            args.read_ceiling = read_ceiling(torch.device("cuda", local_rank))
        fn = {"llama8b": bench_decode, "llama70b": bench_decode, "qwen05b": bench_decode,
              "append": bench_append,
              "prefix": bench_prefix, "continuous": bench_continuous,
              "swap": bench_swap, "mixed": bench_mixed,
              "longprompt": bench_longprompt}[args.workload]
        line = fn(args, rank, world, local_rank)
        if args.workload == "llama8b" and not args.headline_only:
            line.update(sub_benchmarks(args, rank, world, local_rank))
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
