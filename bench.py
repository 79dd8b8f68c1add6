"""Benchmark: effective TFLOPS on kept blocks and ms per forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One step is one block-sparse attention forward of the workload through the
library: the per-tile plan is built from the bool block mask on the GPU and
the tcgen05 attention kernel runs over it (plus the row gather / scatter
kernels when the workload carries a token permutation).  Inputs are resident
in HBM when timing starts; K steps are timed with CUDA events between a
barrier + synchronize on both sides; the max over ranks is reported.

Default workload ``headline``: B1 H16 N16384 D128 bf16 BLOCK128, block mask =
diagonal + Bernoulli(0.10), identity permutation (the "N=16K, D=128, 10%
density" operating point).  With N GPUs every rank runs its own copy of the
workload (weak scaling: 16 heads per rank), with no collective on the path.

``--impl reference`` times the CPU restatement of the reference's block loop
(the oracle port: one float32 numpy program per query block, one process per
host core) on a bounded sample of the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "effective TFLOPS on nonzero blocks & ms/fwd (N=16K, D=128, 10% density), 1/2/4/8 B200"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DTYPE_NAMES = {"torch.bfloat16": "bf16", "torch.float16": "fp16", "torch.float32": "f32"}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary (its ``dram_bytes_per_launch_full: <number>`` line)."""
    p = ROOT / "profiles" / f"attn_tcp_{name}.md"
    if not p.exists():
        return None
    m = re.search(r"dram_bytes_per_launch_full:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons through NVML."""

    REASONS = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x10: "sync_boost",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.idx, self.period = device_index, period_s
        self.samples = []
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.time(), sm, reasons))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()
        return False

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-3:]
        seen = set()
        for _, _, r in win:
            for bit, name in self.REASONS.items():
                if r & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median([s[1] for s in win]) if win else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(win)}


def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def describe(wl) -> str:
    perm = "community-sort permutation" if wl.q_perm is not None else "identity permutation"
    return (f"{wl.name}: B{wl.B} H{wl.H} N{wl.N} D{wl.D} {DTYPE_NAMES[str(wl.dtype)]} BLOCK{wl.block}, "
            f"block density {wl.density:.4f}, {perm}")


def make_cpu_pool(wl):
    """The oracle port of the reference block loop over one head of the
    workload, one process per host core."""
    import numpy as np

    from oracle.cpu_pool import BlockLoopPool

    g = np.random.default_rng(wl.seed)
    q, k, v = (g.standard_normal((wl.N, wl.D), dtype=np.float32) for _ in range(3))
    p_dtype = {"torch.bfloat16": "bfloat16", "torch.float16": "float16"}.get(str(wl.dtype))
    return BlockLoopPool(q, k, v, wl.mask, wl.block, p_dtype)


def cpu_baseline(wl, target_s: float):
    """Whole passes over head 0's query blocks until ``target_s`` of work."""
    with make_cpu_pool(wl) as pool:
        qb = list(range(wl.nb))
        flops, secs, passes = 0.0, 0.0, 0
        while secs < target_s:
            secs += pool.run(qb)
            flops += pool.flops(qb)
            passes += 1
        return {"value": flops / secs / 1e12, "unit": UNIT, "cores": pool.workers, "kind": "port",
                "sample": f"{passes} pass(es) over all {wl.nb} query blocks of one (b,h) head of the workload "
                          f"({secs:.2f} s); float32 numpy port of the reference block loop, one process per core",
                "ms_fwd_extrapolated": 1e3 * secs / passes * wl.B * wl.H}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    from blocksparsefa_reorder_b200 import workloads as W

    wl = W.make(args.workload)
    with make_cpu_pool(wl) as pool:
        all_qb = list(range(wl.nb))
        t_head = pool.run(all_qb)  # calibration pass
        per_step = args.ref_budget_s / (args.steps + args.warmup)
        n_qb = max(1, min(wl.nb, int(wl.nb * per_step / max(t_head, 1e-6))))
        rates, cursor = [], 0
        for i in range(args.warmup + args.steps):
            qb = [(cursor + j) % wl.nb for j in range(n_qb)]
            cursor = (cursor + n_qb) % wl.nb
            dt = pool.run(qb)
            if i >= args.warmup:
                rates.append(pool.flops(qb) / dt / 1e12)
        cores = pool.workers
    v = statistics.median(rates)
    ms_fwd = wl.flops / (v * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_fwd, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mask, q/k/v ~ N(0,1))",
        "config": {"workload": describe(wl)},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{n_qb} query blocks of one (b,h) head per step; float32 numpy port of the "
                                   "reference block loop (the reference has no CPU path of its own), one process "
                                   "per core"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ms_per_step = the workload's kept-block flops at the measured rate",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    from blocksparsefa_reorder_b200 import BlockSparsePlan, block_sparse_attention
    from blocksparsefa_reorder_b200 import workloads as W

    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    wl = W.make(args.workload)
    shard = args.shard_heads and world > 1
    if shard:
        # strong scaling: every rank draws the same full inputs and takes its range of heads
        from blocksparsefa_reorder_b200 import sharding

        ranges = sharding.partition_units(wl.H, world)
        h0, h1 = ranges[rank]
        q, k, v = (t[:, h0:h1] for t in wl.make_qkv(dev))
    else:
        q, k, v = wl.make_qkv(dev, seed=wl.seed + 1000 * rank)
    mask = wl.mask_tensor(dev)
    if shard and mask.dim() == 4 and mask.shape[1] > 1:
        mask = mask[:, h0:h1]
    qp = torch.from_numpy(wl.q_perm).to(dev) if wl.q_perm is not None else None
    kp = torch.from_numpy(wl.kv_perm).to(dev) if wl.kv_perm is not None else None
    o = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    # plan build: one kernel for small masks (<= 4096 tiles, <= 1024 per slice, <= 96 KiB of mask), else
    # count, scan, fill and work order; K and V permutation passes when kv_perm is given (the query
    # permutation is applied inside the attention kernel); the attention kernel
    ms = mask.shape
    slices, nb = (ms[0] * ms[1], ms[-1]) if mask.dim() == 4 else (1, ms[-1])
    tiles_per_slice = (nb * wl.block + 127) // 128
    small = slices * tiles_per_slice <= 4096 and tiles_per_slice <= 1024 and slices * nb * nb <= 96 * 1024
    # (BLOCK 64 launches two forms of the attention kernel; the plan's density picks the one that runs)
    launches_per_step = (1 if small else 4) + (2 if kp is not None else 0) + (2 if wl.block == 64 else 1)
    k_events = []

    def step(record=False):
        plan = BlockSparsePlan(mask, wl.block)
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kv_perm=kp, out=o)
        if record:
            e1.record(stream)
            k_events.append((e0, e1))
        if shard:  # the full output on rank 0 (NCCL point-to-point over NVLink)
            sharding.gather_units(o[0], ranges, dst=0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        time.sleep(0.05)
        barrier(world)
        torch.cuda.synchronize()
        t_wall0 = time.time()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            step(record=True)
        end.record(stream)
        torch.cuda.synchronize()
        t_wall1 = time.time()
        barrier(world)
    ms_step = max_over_ranks(start.elapsed_time(end), world) / args.steps
    kern_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in k_events), world)
    value = wl.flops * (1 if shard else world) / (ms_step * 1e-3) / 1e12
    clocks = clk.summary(t_wall0, t_wall1)

    # e2e: the public API from pinned host buffers, copies inside the timed region.  Every step copies
    # its own inputs host -> device and its output back; steps are pipelined over three streams (step
    # i+1's inputs cross PCIe while step i computes and step i-1's output drains), with two sets of
    # device buffers.
    e2e_steps = max(3, min(args.steps, 10))
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hmask = wl.mask_tensor("cpu").pin_memory()
    hos = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for _ in range(2)]
    hqp = torch.from_numpy(wl.q_perm).pin_memory() if qp is not None else None
    hkp = torch.from_numpy(wl.kv_perm).pin_memory() if kp is not None else None
    hins = [t for t in (hq, hk, hv, hmask, hqp, hkp)]
    dins = [[torch.empty(t.shape, dtype=t.dtype, device=dev) if t is not None else None for t in hins]
            for _ in range(2)]
    douts = [torch.empty_like(o) for _ in range(2)]
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    freed = [None, None]  # compute of the step that last used buffer set b is done
    drained = [None, None]  # d2h of the step that last used output buffer b is done

    def e2e_run(nsteps):
        for i in range(nsteps):
            b = i % 2
            with torch.cuda.stream(s_h2d):
                if freed[b] is not None:
                    s_h2d.wait_event(freed[b])
                for d, h in zip(dins[b], hins):
                    if d is not None:
                        d.copy_(h, non_blocking=True)
                loaded = ev()
                loaded.record(s_h2d)
            stream.wait_event(loaded)
            if drained[b] is not None:
                stream.wait_event(drained[b])
            dq, dk, dv, dm, dqp, dkp = dins[b]
            block_sparse_attention(dq, dk, dv, dm, block=wl.block, q_perm=dqp, kv_perm=dkp, out=douts[b])
            freed[b] = ev()
            freed[b].record(stream)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(freed[b])
                hos[b].copy_(douts[b], non_blocking=True)
                drained[b] = ev()
                drained[b].record(s_d2h)
        stream.wait_stream(s_d2h)
        stream.wait_stream(s_h2d)

    e2e_run(2)
    torch.cuda.synchronize()
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    s_h2d.wait_stream(stream)
    e2e_run(e2e_steps)
    e2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e2e_steps, world)
    ho = hos[0]
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hmask))
    h2d += sum(t.numel() * t.element_size() for t in (hqp, hkp) if t is not None)
    d2h = ho.numel() * ho.element_size()
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    local_flops = wl.flops * (h1 - h0) / wl.H if shard else wl.flops
    achieved = local_flops / (kern_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if shard else "weak",
        "vs_baseline": None, "dtype": DTYPE_NAMES[str(wl.dtype)],
        "data": "synthetic: seeded block mask; q, k, v ~ N(0,1) drawn on the device",
        "config": {"workload": describe(wl), "B": wl.B, "H_per_rank": (h1 - h0) if shard else wl.H, "N": wl.N,
                   "D": wl.D,
                   "block": wl.block, "nnz_blocks_per_rank": wl.nnz_blocks, "density": round(wl.density, 5),
                   "flops_per_rank": wl.flops / world if shard else wl.flops,
                   "parallelism": (f"heads sharded over {world} ranks, O gathered to rank 0 by NCCL point-to-point "
                                   f"inside the step" if shard else f"(b,h) units, {world} rank(s), no collective"),
                   "l2": "inputs larger than L2 (q, k, v, o = %d MiB per rank); no flush" %
                         (4 * q.numel() * q.element_size() // 2**20)},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": profile_traffic(wl.name),
                     "kernel": "attn_tcp_kernel", "kernel_ms": kern_ms,
                     "peak_source": f"bf16_tflops (burst) of {peak_kind} peaks"},
        "e2e": {"value": wl.flops * (1 if shard else world) / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "block_sparse_attention(q, k, v, mask) from pinned host buffers; per step H2D of "
                        "q, k, v, mask (+perms) and D2H of o, pipelined across steps on copy streams"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        cb = cpu_baseline(wl, args.cpu_seconds)
        cb.pop("ms_fwd_extrapolated", None)
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="headline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    ap.add_argument("--ref-budget-s", type=float, default=90.0, help="total CPU time of the reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard-heads", action="store_true",
                    help="under torchrun: split the workload's heads over the ranks (strong scaling) and gather "
                         "O to rank 0 inside each step, as the long-context configuration specifies")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
