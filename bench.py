"""Benchmark: effective TFLOPS on kept blocks and ms per forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--scaling strong|weak] [--no-per-config]

One step is one block-sparse attention forward of the workload through the
library: the tcgen05 attention kernel over the per-tile plan of the block
mask (plus the K / V row-permutation kernels when the workload carries a
token permutation; the query permutation is applied inside the attention
kernel).  As in the reference's timed loop (BlockSparseTriton_Naive.py:
131-161 reuses one block mask for every iteration), the plan is built once per
mask before timing; the plan build is timed on its own and a second number
rebuilds it every step.  The steps are replayed from CUDA graphs of the call
(the same kernels the eager call launches, without per-step host work): a
graph of 8 (or more, whole rotations over the input copies) forwards back to
back, then single-forward graphs for the remainder, so that exactly K
forwards run; the attention kernel's own time is taken from events around
single-forward replays.
Inputs are resident in HBM when timing starts; when one rank's inputs would
fit in L2 the steps rotate over several input copies so that every step reads
from DRAM.  K steps are timed with CUDA events between a barrier + synchronize
on both sides; the max over ranks is reported.

Default workload ``headline``: B1 H16 N16384 D128 bf16 BLOCK128, block mask
= diagonal + Bernoulli(0.10), identity permutation (the "N=16K, D=128, 10%
density" operating point).  Under torchrun the (b, h) units of the workload
are split over the ranks (strong scaling, no collective; ``--scaling weak``
gives every rank its own copy instead, and the strong run also reports the
weak number).  The long-context workload gathers O to rank 0 inside the step
(NCCL point-to-point over NVLink), as that configuration specifies.

At N = 1 the line also carries ``per_config``: every benchmark configuration
measured on this GPU (kernel time, TFLOP/s, roofline fractions, measured
density, a max-abs-error spot check against an fp64 masked softmax on sampled
query blocks).

At N = 1 the line also carries ``gpu_comparator``: ``torch.compile(
flex_attention)`` (the reference's FlexAttention backend, library code) on the
same inputs and block mask on this GPU, with this library's speed-up over it.

``--impl reference`` times the CPU restatement of the reference's block loop
(the oracle port: one float32 numpy program per query block, one process per
host core) on a bounded sample of the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
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
L2_BYTES = 126 * 2**20
CONFIGS = ["plumbing", "random", "sbm", "headline", "longctx", "sweep_p01", "sweep_p05", "sweep_p20", "sweep_p50"]
# long context under torchrun: each rank's heads are computed in this many
# parts, each part's O sent to rank 0 while the next part computes
GATHER_PARTS = 4
# DRAM bytes per attention launch from one ncu capture of the same kernel on the
# same workload (dram__bytes_read.sum + dram__bytes_write.sum), with the
# command that produced it; --ncu-csv takes the figure from a capture instead.
NCU_TRAFFIC = {
    "headline": (249925376.0, "ncu --set full --clock-control none -k regex:attn_tcp -s 3 -c 1 python bench.py "
                              "--steps 10 --warmup 3 --no-cpu-baseline --no-per-config --sustained-seconds 0 "
                              "(headline workload)"),
    "sweep_p20": (4038844416.0, "ncu --set full --clock-control none -k regex:attn_tcp -s 24 -c 2 python bench.py "
                                "--workload sweep_p20 --units 8 --steps 5 --warmup 3 --no-cpu-baseline "
                                "--no-per-config --sustained-seconds 0 --no-backward --no-gpu-comparator, DRAM bytes "
                                "of the 8-unit launch x 16 (the 128 units are independent)"),
    "sweep_p01": (4005896192.0, "ncu --set full --clock-control none -k regex:attn_tcp -s 24 -c 2 python bench.py "
                                "--workload sweep_p01 --units 8 --steps 5 --warmup 3 --no-cpu-baseline "
                                "--no-per-config --sustained-seconds 0 --no-backward --no-gpu-comparator, DRAM bytes "
                                "of the 8-unit launch x 16 (the 128 units are independent)"),
}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def ncu_csv_traffic(path):
    """dram__bytes_read.sum + dram__bytes_write.sum of the first attention
    launch in an ``ncu --page raw --csv`` export."""
    import csv

    rows = list(csv.reader(open(path)))
    hdr = rows[0]
    ir, iw, ik = (hdr.index(c) for c in ("dram__bytes_read.sum", "dram__bytes_write.sum", "Kernel Name"))
    units = rows[1]
    scale = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    for r in rows[2:]:
        if "attn_tcp" in r[ik]:
            return float(r[ir]) * scale.get(units[ir], 1.0) + float(r[iw]) * scale.get(units[iw], 1.0)
    return None


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons through NVML."""

    REASONS = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x10: "sync_boost",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.005):
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

    def summary(self, t0: float, t1: float, what: str):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-3:]
        seen = set()
        for _, _, r in win:
            for bit, name in self.REASONS.items():
                if r & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median([s[1] for s in win]) if win else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(win), "window": what}


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


def config_dict(wl, world: int, scaling: str) -> dict:
    """The workload as both arms print it (the same dict for the same run)."""
    from blocksparsefa_reorder_b200.sharding import partition_units

    units = wl.B * wl.H
    per_rank = max(b - a for a, b in partition_units(units, world)) if scaling == "strong" else units
    return {"workload": describe(wl), "B": wl.B, "H": wl.H, "N": wl.N, "D": wl.D, "block": wl.block,
            "dtype": DTYPE_NAMES[str(wl.dtype)], "density": round(wl.density, 5), "nnz_blocks": wl.nnz_blocks,
            "flops_per_forward": wl.flops, "permutation": wl.q_perm is not None,
            "parallelism": (f"(b,h) units split over {world} rank(s), at most {per_rank} per rank"
                            if scaling == "strong" else f"each of {world} rank(s) runs the whole workload")
                           + ("; O gathered to rank 0 by NCCL point-to-point inside the step"
                              if wl.name == "longctx" and scaling == "strong" and world > 1 else "; no collective")}


def scaling_of(world: int, requested: str) -> str:
    return "strong" if world > 1 and requested == "strong" else "weak"


# ----------------------------------------------------------------------------- inputs and work
def unit_slice(t, lo, hi):
    """Units [lo, hi) of a [B, H, ...] tensor as [1, hi - lo, ...] (the whole tensor when all)."""
    B, H = t.shape[:2]
    if lo == 0 and hi == B * H:
        return t
    return t.reshape((B * H,) + tuple(t.shape[2:]))[lo:hi].unsqueeze(0)


def algorithmic_bytes(wl, units: int) -> float:
    """Q read + O write once, each head's kept key blocks of K and V once
    (shared through L2 by the tiles of the head), and the plan (tile_ptr,
    tile_order, at most one entry per kept block)."""
    import numpy as np

    elt = 4 if DTYPE_NAMES[str(wl.dtype)] == "f32" else 2
    cols = np.nonzero(wl.mask.any(axis=0))[0]
    key_rows = int(sum(min(wl.block, wl.N - j * wl.block) for j in cols))
    T = (wl.nb * wl.block + 127) // 128
    plan = 4 * (2 * T + 1 + int(wl.mask.sum()))
    return float(elt * units * (2 * wl.N * wl.D + 2 * key_rows * wl.D) + plan)


class Runner:
    """A workload's units [lo, hi) resident on this GPU, its plan built once,
    a CUDA graph of one forward per input copy, and one graph of ``group``
    forwards back to back (whole rotations over the copies, at least
    ``batch``), which the timed loops replay so that consecutive forwards are
    not separated by a graph launch each."""

    def __init__(self, wl, dev, lo, hi, seed=None, copies=None, graphs=True, kernel="auto", batch=8):
        import torch

        from blocksparsefa_reorder_b200 import BlockSparsePlan

        self.wl, self.dev, self.lo, self.hi = wl, dev, lo, hi
        self.kernel = kernel if str(wl.dtype) != "torch.float32" else "auto"
        self.units = hi - lo
        q, k, v = (unit_slice(t, lo, hi).contiguous() for t in wl.make_qkv(dev, seed=seed))
        self.mask = wl.mask_tensor(dev)
        self.plan = BlockSparsePlan(self.mask, wl.block)
        self.qp = torch.from_numpy(wl.q_perm).to(dev) if wl.q_perm is not None else None
        self.kp = torch.from_numpy(wl.kv_perm).to(dev) if wl.kv_perm is not None else None
        per_copy = 4 * q.numel() * q.element_size()
        if copies is None:
            copies = min(32, max(1, math.ceil(2 * L2_BYTES / per_copy)))
        self.sets = [(q, k, v, torch.empty_like(q))]
        for _ in range(copies - 1):
            self.sets.append((q.clone(), k.clone(), v.clone(), torch.empty_like(q)))
        self.footprint = per_copy * copies
        self.graphs = []
        self.batched, self.group = None, 1
        # warm the host-side caches and the kernels once per copy, then capture
        for s in self.sets:
            self.forward(s)
        torch.cuda.synchronize(dev)
        if graphs:
            for s in self.sets:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.forward(s)
                self.graphs.append(g)
            self.group = copies * max(1, math.ceil(batch / copies))
            self.batched = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.batched):
                for i in range(self.group):
                    self.forward(self.sets[i % copies])
            self.batched.replay()  # first launch (graph upload) outside any timed region
            torch.cuda.synchronize(dev)

    def forward(self, s):
        from blocksparsefa_reorder_b200 import block_sparse_attention

        q, k, v, o = s
        return block_sparse_attention(q, k, v, plan=self.plan, q_perm=self.qp, kv_perm=self.kp, out=o,
                                      kernel=self.kernel)

    def step(self, i):
        if self.graphs:
            self.graphs[i % len(self.graphs)].replay()
        else:
            self.forward(self.sets[i % len(self.sets)])

    def run_steps(self, n):
        """Exactly n forwards: whole replays of the batched graph, then single ones."""
        full, rest = divmod(n, self.group) if self.batched is not None else (0, n)
        for _ in range(full):
            self.batched.replay()
        for i in range(rest):
            self.step(i)

    @property
    def flops(self):
        return self.wl.flops * self.units / (self.wl.B * self.wl.H)

    def launches_per_step(self):
        n = 2 if self.wl.block == 64 else 1  # BLOCK 64: both kernel forms launch, the plan picks one
        return n + (2 if self.kp is not None else 0)

    def release(self):
        self.graphs = []
        self.batched = None
        self.sets = []


def time_steps(run, steps, stream, world, per_step_events=False):
    """Time ``steps`` steps between barrier + synchronize; returns (ms per
    step max over ranks, per-step event durations on this rank)."""
    import torch

    evs = []
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        if per_step_events:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run(i)
            e1.record(stream)
            evs.append((e0, e1))
        else:
            run(i)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    return max_over_ranks(ms, world), [a.elapsed_time(b) for a, b in evs]


def time_block(run_n, steps, stream, world):
    """Time ``run_n(steps)`` (all steps issued at once) between barrier +
    synchronize; ms per step, max over ranks."""
    import torch

    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    run_n(steps)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end) / steps, world)


def time_plan(plan, mask, stream, reps=20):
    """Mean device time of one plan build (into the plan's own buffers)."""
    import torch

    for _ in range(3):
        plan.update(mask)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        plan.update(mask)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def spot_check(wl, o, q, k, v, unit, qblocks):
    """Max |o - fp64 masked softmax| over the rows of the given query blocks
    (new token order) of one (b, h) unit, computed on the host."""
    import numpy as np
    import torch

    def host(t):
        return t.reshape((-1,) + tuple(t.shape[2:]))[unit].double().cpu()

    qh, kh, vh, oh = (host(t) for t in (q, k, v, o))
    if wl.kv_perm is not None:
        kp = torch.from_numpy(wl.kv_perm)
        kh, vh = kh[kp], vh[kp]
    scale = 1.0 / math.sqrt(wl.D)
    err = 0.0
    for mb in qblocks:
        r0, r1 = mb * wl.block, min(wl.N, (mb + 1) * wl.block)
        rows = torch.arange(r0, r1) if wl.q_perm is None else torch.from_numpy(wl.q_perm[r0:r1])
        cols = np.nonzero(wl.mask[mb])[0]
        if cols.size == 0:
            ref = torch.zeros(r1 - r0, wl.D, dtype=torch.float64)
        else:
            keys = torch.from_numpy(np.concatenate([np.arange(j * wl.block, min(wl.N, (j + 1) * wl.block))
                                                    for j in cols]))
            s = (qh[rows] @ kh[keys].T) * scale
            ref = torch.softmax(s, dim=-1) @ vh[keys]
        err = max(err, float((oh[rows] - ref).abs().max()))
    return err


# ----------------------------------------------------------------------------- CPU baselines
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
                          f"({secs:.2f} s); float32 numpy port of the reference block loop, one process per core"}


def cpu_dense_masked(wl, target_s: float):
    """The dense-masked softmax attention in PyTorch on the host (float32,
    every host thread): S = QK^T * scale over all keys, -inf outside the block
    mask, softmax, PV, over query-row chunks of one head until ``target_s``;
    reported as effective TFLOPS on the kept blocks it covered."""
    import torch

    from oracle.cpu_pool import host_cores

    cores = host_cores()
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(wl.seed)
    q, k, v = (torch.randn(wl.N, wl.D, generator=g) for _ in range(3))
    mask = torch.from_numpy(wl.mask)
    scale = 1.0 / math.sqrt(wl.D)
    bpc = max(1, 1024 // wl.block)
    secs, flops, blocks_done, mb = 0.0, 0.0, 0, 0
    while secs < target_s and mb < wl.nb:
        m = mask[mb:mb + bpc]
        r0, r1 = mb * wl.block, min(wl.N, (mb + m.shape[0]) * wl.block)
        tm = m.repeat_interleave(wl.block, 0).repeat_interleave(wl.block, 1)[: r1 - r0, :wl.N]
        t0 = time.perf_counter()
        s = (q[r0:r1] @ k.T) * scale
        s.masked_fill_(~tm, float("-inf"))
        p = torch.nan_to_num(torch.softmax(s, dim=-1))
        o = p @ v
        secs += time.perf_counter() - t0
        flops += 4.0 * wl.block * wl.block * wl.D * int(m.sum())
        blocks_done += m.shape[0]
        mb += bpc
        del o
    return {"value": flops / secs / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{blocks_done} of {wl.nb} query blocks of one (b,h) head ({secs:.2f} s); dense masked "
                      f"softmax attention in float32 PyTorch on the host (all keys scored, -inf outside the mask)",
            "ms_per_forward_extrapolated": 1e3 * secs * wl.nb / max(1, blocks_done) * wl.B * wl.H}


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    from blocksparsefa_reorder_b200 import workloads as W

    wl = W.make(args.workload)
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    scaling = scaling_of(world, args.scaling)
    with make_cpu_pool(wl) as pool:
        all_qb = list(range(wl.nb))
        t_head = pool.run(all_qb)  # calibration pass
        per_step = args.ref_budget_s / (args.steps + args.warmup)
        n_qb = max(1, min(wl.nb, int(wl.nb * per_step / max(t_head, 1e-6))))
        rates, times, cursor = [], [], 0
        for i in range(args.warmup + args.steps):
            qb = [(cursor + j) % wl.nb for j in range(n_qb)]
            cursor = (cursor + n_qb) % wl.nb
            dt = pool.run(qb)
            if i >= args.warmup:
                rates.append(pool.flops(qb) / dt / 1e12)
                times.append(dt)
        cores = pool.workers
    v = statistics.median(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mask, q/k/v ~ N(0,1))",
        "config": config_dict(wl, world, scaling),
        "step": f"{n_qb} query blocks of one (b,h) head of the workload (the measured sample)",
        "ms_per_forward_extrapolated": wl.flops / (v * 1e12) * 1e3,
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{n_qb} query blocks of one (b,h) head per step; float32 numpy port of the "
                                   "reference block loop (the reference has no CPU path of its own), one process "
                                   "per core"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- per-config measurement
def measure_config(name, dev, peaks, steps=10, warmup=3, kernel="auto"):
    """One benchmark configuration on this GPU (the whole workload)."""
    import torch

    from blocksparsefa_reorder_b200 import block_sparse_attention, permute_rows
    from blocksparsefa_reorder_b200 import workloads as W

    wl = W.make(name)
    units = wl.B * wl.H
    stream = torch.cuda.current_stream(dev)
    run = Runner(wl, dev, 0, units, kernel=kernel)
    for i in range(warmup):
        run.step(i)
    kernel_call, extra = run.step, None
    if run.kp is not None:
        # the attention kernel alone: K and V already in the new order, the
        # query permutation (fused into the kernel) still applied
        q, k, v, o = run.sets[0]
        k2 = permute_rows(k, run.kp, dim=2, inverse=False)
        v2 = permute_rows(v, run.kp, dim=2, inverse=False)

        def call():
            block_sparse_attention(q, k2, v2, plan=run.plan, q_perm=run.qp, out=o, kernel=run.kernel)

        call()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            call()
        for _ in range(warmup):
            g.replay()
        kernel_call, extra = (lambda i: g.replay()), (g, k2, v2)
    # the kernel alone first, then the whole steps, with the SM clock of each
    with ClockSampler(dev.index if dev.index is not None else 0, period_s=0.001) as clk:
        t0 = time.time()
        _, evs = time_steps(kernel_call, steps, stream, 1, per_step_events=True)
        t1 = time.time()
        step_ms = time_block(run.run_steps, steps, stream, 1)
        t2 = time.time()
    kern_ms = statistics.mean(evs)
    ck, cs = clk.summary(t0, t1, "kernel"), clk.summary(t1, t2, "step")
    clocks = {"kernel_sm_mhz": ck["sm_mhz"], "step_sm_mhz": cs["sm_mhz"],
              "reasons": sorted(set(ck["reasons"]) | set(cs["reasons"]))}
    del extra
    # correctness spot check of the whole step's output
    run.step(0)
    torch.cuda.synchronize()
    q0, k0, v0, o0 = run.sets[0]
    qbs = sorted({0, wl.nb // 2, wl.nb - 1})
    err = max(spot_check(wl, o0, q0, k0, v0, u, qbs) for u in (0, units - 1))
    t_plan = time_plan(run.plan, run.mask, stream)
    tile_entries = run.plan.nnz_entries()
    tiles = run.plan.mask_b * run.plan.mask_h * run.plan.tiles_per_row
    flops = wl.flops
    nbytes = algorithmic_bytes(wl, units)
    tensor = wl.dtype != torch.float32
    tf = flops / (kern_ms * 1e-3) / 1e12
    gbs = nbytes / (kern_ms * 1e-3) / 1e9
    peak_tf = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    peak_bw = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    t_tensor, t_hbm = flops / (peak_tf * 1e12), nbytes / (peak_bw * 1e9)
    bound = ("tensor" if t_tensor >= t_hbm else "hbm") if tensor else "cuda-core fp32 (correctness path)"
    out = {
        "workload": describe(wl), "density": round(wl.density, 5), "nnz_blocks": wl.nnz_blocks,
        "kernel": ("attn_simt_kernel" if not tensor else
                   "attn_tcp_kernel " + ("paired" if wl.block == 64 and tile_entries >= 4 * tiles else
                                         "single-block steps" if wl.block == 64 else "BLOCK128")),
        "entries_per_tile": round(tile_entries / tiles, 2),
        "kernel_ms": kern_ms, "step_ms": step_ms, "plan_build_ms": t_plan,
        "tflops_kernel": tf, "tflops_step": flops / (step_ms * 1e-3) / 1e12,
        "bound": bound,
        "tensor_frac": tf / peak_tf if tensor else None,
        "hbm_gbs": gbs, "hbm_frac": gbs / peak_bw,
        "algorithmic_bytes": nbytes, "algorithmic_flops": flops,
        "max_abs_err": err, "err_check": "fp64 masked softmax on the host, query blocks %s of (b,h) units 0 and %d"
                                         % (qbs, units - 1),
        "clocks": clocks,
    }
    if name in NCU_TRAFFIC:
        out["traffic"], out["traffic_source"] = NCU_TRAFFIC[name][0], "committed ncu capture: " + NCU_TRAFFIC[name][1]
    run.release()
    del run
    torch.cuda.empty_cache()
    return out


def measure_flex(wl, dev, steps, warmup=5):
    """GPU comparator on the same B200: ``torch.compile(flex_attention)``
    with a BlockMask of the workload's block mask, the reference's
    FlexAttention backend (BlockSparseXF.py:43-63) and the comparator BASELINE
    names for every configuration.  Library code, not this build: timed with
    CUDA events over ``steps`` calls after ``warmup``, outputs compared with
    this library's on the same inputs."""
    import torch
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    from blocksparsefa_reorder_b200 import BlockSparsePlan, block_sparse_attention

    if wl.q_perm is not None or wl.kv_perm is not None or wl.dtype == torch.float32:
        return {"skipped": "comparator run on identity-permutation 16-bit workloads only"}
    q, k, v = wl.make_qkv(dev)
    bm = torch.from_numpy(wl.mask).to(dev)
    blk = wl.block

    def mask_mod(b, h, qi, ki):
        return bm[qi // blk, ki // blk]

    # its kernel tiles must divide the mask's block (64-blocks need 64 x 64 tiles)
    opts = {"BLOCK_M": blk, "BLOCK_N": blk} if blk < 128 else None
    t0 = time.time()
    block_mask = create_block_mask(mask_mod, None, None, wl.N, wl.N, device=dev, BLOCK_SIZE=blk)
    fa = torch.compile(flex_attention)
    o_f = fa(q, k, v, block_mask=block_mask, kernel_options=opts)
    torch.cuda.synchronize()
    setup_s = time.time() - t0
    o = block_sparse_attention(q, k, v, plan=BlockSparsePlan(wl.mask_tensor(dev), blk))
    diff = (o.float() - o_f.float()).abs().max().item()
    for _ in range(warmup):
        fa(q, k, v, block_mask=block_mask, kernel_options=opts)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fa(q, k, v, block_mask=block_mask, kernel_options=opts)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    out = {"impl": "torch.compile(flex_attention) with a BlockMask of the same block mask (BLOCK_SIZE %d)" % blk,
           "value": wl.flops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
           "max_abs_diff_vs_this_library": diff, "setup_s": setup_s,
           "what": "secondary GPU comparator on the same B200; the reference arm stays the CPU path"}
    del q, k, v, o, o_f, block_mask
    torch.cuda.empty_cache()
    return out


def measure_backward(wl, dev, steps):
    """The backward pass on the workload (no permutation, 16-bit): device
    time of one block_sparse_attention_backward call (Delta, dQ, dK / dV
    kernels) with the forward's o / lse and both plans resident, against the
    usual 2.5x-forward flop count (5 GEMMs of the kept blocks)."""
    import torch

    from blocksparsefa_reorder_b200 import (BlockSparsePlan, block_sparse_attention,
                                            block_sparse_attention_backward, transposed_plan)

    if wl.q_perm is not None or str(wl.dtype) == "torch.float32":
        return None
    q, k, v = wl.make_qkv(dev)
    g = torch.Generator(device="cpu").manual_seed(wl.seed + 7)
    dout = torch.randn(q.shape, generator=g).to(q.dtype).to(dev)
    m = wl.mask_tensor(dev)
    plan = BlockSparsePlan(m, wl.block)
    plan_t = transposed_plan(plan, m)
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    for _ in range(3):
        block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=plan_t)
    stream = torch.cuda.current_stream(dev)
    _, evs = time_steps(lambda i: block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=plan_t),
                        max(3, min(steps, 20)), stream, 1, per_step_events=True)
    ms = statistics.median(evs)
    peaks, _ = load_peaks()
    tf = 2.5 * wl.flops / (ms * 1e-3) / 1e12
    return {"ms": ms, "tflops": tf, "frac": tf / float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])),
            "flops_counted": 2.5 * wl.flops,
            "what": "dq, dk, dv of the workload from dout (bf16): Delta, dQ and dK/dV kernels, P recomputed from the "
                    "forward's lse; flops counted as 2.5 x the forward's (the kernels recompute S and dP in both "
                    "gradient kernels, 3.5 x)"}


# ----------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    from blocksparsefa_reorder_b200 import block_sparse_attention, sharding
    from blocksparsefa_reorder_b200 import workloads as W

    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    wl = W.make(args.workload)
    peaks, peak_kind = load_peaks()
    units_total = wl.B * wl.H
    scaling = scaling_of(world, args.scaling)
    strong = scaling == "strong"
    if args.units:
        # a smaller case of the same kernel (ncu captures): the first U (b, h)
        # units of the workload on every rank
        strong, scaling = False, "weak"
        ranges = [(0, min(args.units, units_total))] * world
    else:
        ranges = sharding.partition_units(units_total, world) if strong else [(0, units_total)] * world
    lo, hi = ranges[rank]
    gather = strong and wl.name == "longctx"
    run = Runner(wl, dev, lo, hi, seed=None if strong or world == 1 else wl.seed + 1000 * rank,
                 graphs=not gather, kernel=args.kernel)
    per_rank_flops = run.flops
    job_flops = wl.flops if strong else per_rank_flops * world

    if gather:
        # long context: each rank's heads in GATHER_PARTS parts; a part's O
        # goes to rank 0 (placed at its global head index) while the next
        # part computes, so only the last part's transfer is exposed
        q, k, v, o = run.sets[0]
        full = torch.empty((units_total, wl.N, wl.D), dtype=q.dtype, device=dev) if rank == 0 else None

        parts = sharding.split_parts(ranges, GATHER_PARTS)

        def step(i):
            works = []
            for pieces, offs in parts:
                a, b = pieces[rank]
                if b > a:
                    block_sparse_attention(q[:, a:b], k[:, a:b], v[:, a:b], plan=run.plan, out=o[:, a:b],
                                           kernel=run.kernel)
                _, w = sharding.gather_units(o[0, a:b], pieces, dst=0, async_op=True, out=full, offsets=offs)
                works += w
            for w in works:
                w.wait()
    else:
        step = run.step

    def run_n(n):
        if gather:
            for i in range(n):
                step(i)
        else:
            run.run_steps(n)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # the timed region follows the warm-up directly (clocks at their burst
    # level); NVML is sampled every millisecond through it.  The attention
    # kernel's own time comes from events around single steps right after.
    with ClockSampler(local, period_s=0.001) as clk:
        t_wall0 = time.time()
        ms_step = time_block(run_n, args.steps, stream, world)
        t_wall1 = time.time()
        _, evs = time_steps(step, args.steps, stream, world, per_step_events=True)
    kern_single = max_over_ranks(statistics.mean(evs), world)
    # When a step is exactly one attention launch (no permutation passes, no
    # gather), the timed region's ms per step is that kernel's average launch
    # duration (launches back to back from graphs, the gaps between them
    # included); otherwise the events around single-step replays.
    one_launch = not gather and run.launches_per_step() == 1
    kern_ms = ms_step if one_launch else kern_single
    kern_src = ("timed region: one attention launch per step, back to back from CUDA graphs (average launch "
                "duration, gaps included)" if one_launch else "CUDA events around single-step replays on the "
                "launching stream")
    value = job_flops / (ms_step * 1e-3) / 1e12
    clocks = clk.summary(t_wall0, t_wall1, "timed region")

    # plan rebuilt every step (into the same buffers), timed right after the
    # main steps, at the same clocks
    def step_with_plan(i):
        run.plan.update(run.mask)
        run.forward(run.sets[i % len(run.sets)])

    ms_plan_step, plan_how = None, None
    if not gather:
        # the plan build and the forward of a step captured together, one
        # graph per input copy (the same kernels the eager calls launch)
        plan_graphs = []
        try:
            for sset in run.sets:
                run.plan.update(run.mask)
                run.forward(sset)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    run.plan.update(run.mask)
                    run.forward(sset)
                plan_graphs.append(g)
            plan_step = lambda i: plan_graphs[i % len(plan_graphs)].replay()  # noqa: E731
            plan_how = "plan rebuilt from the mask every step: plan build and forward replayed from one CUDA graph"
        except Exception as e:  # not capturable here: eager calls instead
            plan_graphs = []
            plan_step = step_with_plan
            plan_how = f"plan rebuilt from the mask every step (eager calls; graph capture failed: {type(e).__name__})"
        for i in range(3):
            plan_step(i)
        ms_plan_step, _ = time_steps(plan_step, args.steps, stream, world)
        del plan_graphs
    # the same steps after ~sustained_seconds of continuous load (power cap
    # reached), against the sustained peak
    sustained = None
    if args.sustained_seconds > 0:
        t_one, _ = time_steps(step, 3, stream, world)
        n_load = max(1, int(args.sustained_seconds * 1e3 / max(t_one, 1e-3)))
        with ClockSampler(local, period_s=0.005) as clk_s:
            run_n(n_load)
            torch.cuda.synchronize()
            ts0 = time.time()
            ms_s = time_block(run_n, args.steps, stream, world)
            ts1 = time.time()
            _, evs_s = time_steps(step, args.steps, stream, world, per_step_events=True)
        kern_s = ms_s if one_launch else max_over_ranks(statistics.mean(evs_s), world)
        sus_peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        ach_s = per_rank_flops / (kern_s * 1e-3) / 1e12
        sustained = {"value": job_flops / (ms_s * 1e-3) / 1e12, "ms_per_step": ms_s,
                     "kernel_ms": kern_s, "achieved": ach_s, "peak": sus_peak, "frac": ach_s / sus_peak,
                     "peak_source": f"bf16_tflops_sustained of {peak_kind} peaks",
                     "what": "the same steps timed after %.1f s of identical steps (%d) without a pause"
                             % (args.sustained_seconds, n_load),
                     "clocks": clk_s.summary(ts0, ts1, "timed region"),
                     "clocks_load": clk_s.summary(ts0 - args.sustained_seconds, ts0, "the load before it")}

    t_plan = time_plan(run.plan, run.mask, stream)

    # the weak-scaling number beside the strong one
    weak = None
    if strong and not gather:
        run_w = Runner(wl, dev, 0, units_total, seed=wl.seed + 1000 * rank, kernel=args.kernel)
        for i in range(3):
            run_w.step(i)
        ms_w = time_block(run_w.run_steps, args.steps, stream, world)
        weak = {"value": wl.flops * world / (ms_w * 1e-3) / 1e12, "ms_per_step": ms_w,
                "what": "every rank runs the whole workload on its own inputs (replicas), no collective"}
        run_w.release()
        del run_w

    # e2e: the public API from pinned host buffers, copies inside the timed
    # region.  Every step copies its own inputs host -> device and its output
    # back; steps are pipelined over copy streams (step i+1's inputs cross PCIe
    # while step i computes and step i-1's output drains), with two sets of
    # device buffers.
    q, k, v, o = run.sets[0]
    e2e_steps = max(3, min(args.steps, 10))
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hmask = wl.mask_tensor("cpu").pin_memory()
    hos = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for _ in range(2)]
    hqp = torch.from_numpy(wl.q_perm).pin_memory() if run.qp is not None else None
    hkp = torch.from_numpy(wl.kv_perm).pin_memory() if run.kp is not None else None
    hins = [hq, hk, hv, hmask, hqp, hkp]
    dins = [[torch.empty(t.shape, dtype=t.dtype, device=dev) if t is not None else None for t in hins]
            for _ in range(2)]
    douts = [torch.empty_like(o) for _ in range(2)]
    # host -> device copies spread over two streams (two copy engines share
    # the PCIe link), device -> host on a third
    s_h2d, s_h2d2, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    freed = [None, None]
    drained = [None, None]

    def e2e_run(nsteps):
        for i in range(nsteps):
            b = i % 2
            pairs = [(d, h) for d, h in zip(dins[b], hins) if d is not None]
            for j, s_c in enumerate((s_h2d, s_h2d2)):
                with torch.cuda.stream(s_c):
                    if freed[b] is not None:
                        s_c.wait_event(freed[b])
                    for d, h in pairs[j::2]:
                        d.copy_(h, non_blocking=True)
                    loaded = ev()
                    loaded.record(s_c)
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
        stream.wait_stream(s_h2d2)

    e2e_run(2)
    torch.cuda.synchronize()
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    s_h2d.wait_stream(stream)
    s_h2d2.wait_stream(stream)
    e2e_run(e2e_steps)
    e2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e2e_steps, world)
    h2d = sum(t.numel() * t.element_size() for t in hins if t is not None)
    d2h = hos[0].numel() * hos[0].element_size()
    barrier(world)
    footprint, n_copies, group = run.footprint, len(run.sets), run.group
    launches = run.launches_per_step()
    run.release()
    del run, q, k, v, o, dins, douts
    torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    backward = measure_backward(wl, dev, args.steps) if world == 1 and not args.no_backward else None

    gpu_comparator = None
    if world == 1 and not args.no_gpu_comparator:
        try:
            gpu_comparator = measure_flex(wl, dev, args.steps)
        except Exception as e:  # report, do not hide
            gpu_comparator = {"error": f"{type(e).__name__}: {e}"}

    per_config = None
    if world == 1 and not args.no_per_config:
        per_config = {}
        for name in args.configs.split(","):
            try:
                per_config[name] = measure_config(name, dev, peaks, kernel=args.kernel)
            except Exception as e:  # report, do not hide
                per_config[name] = {"error": f"{type(e).__name__}: {e}"}
                continue
            if args.no_gpu_comparator:
                continue
            try:
                fc = measure_flex(W.make(name), dev, steps=5, warmup=3)
                if "ms_per_step" in fc:
                    fc = {"flex_ms": fc["ms_per_step"], "flex_tflops": fc["value"],
                          "this_library_speedup": fc["ms_per_step"] / per_config[name]["kernel_ms"],
                          "max_abs_diff": fc["max_abs_diff_vs_this_library"]}
                per_config[name]["gpu_comparator"] = fc
            except Exception as e:  # report, do not hide
                per_config[name]["gpu_comparator"] = {"error": f"{type(e).__name__}: {e}"}

    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    achieved = per_rank_flops / (kern_ms * 1e-3) / 1e12
    traffic, traffic_src = None, None
    if args.ncu_csv:
        traffic, traffic_src = ncu_csv_traffic(args.ncu_csv), f"ncu capture {args.ncu_csv}"
    elif wl.name in NCU_TRAFFIC and world == 1:
        traffic, traffic_src = NCU_TRAFFIC[wl.name][0], "committed ncu capture: " + NCU_TRAFFIC[wl.name][1]
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": DTYPE_NAMES[str(wl.dtype)],
        "data": "synthetic: seeded block mask; q, k, v ~ N(0,1) drawn on the device",
        "config": dict(config_dict(wl, world, scaling), **({"units_timed": ranges[0][1]} if args.units else {})),
        "setup": {
            "units_per_rank": [b - a for a, b in ranges],
            "step": "attention forward with the plan built once per mask (the reference's timed loop reuses "
                    "its block mask); the K steps are replayed from CUDA graphs of %d forwards back to back "
                    "(then single-forward graphs for the remainder), exactly K forwards" % group if not gather else
                    "attention forward in %d parts of the rank's heads with the O gather to rank 0 posted "
                    "after each part (eager calls)" % GATHER_PARTS,
            "l2": ("inputs larger than L2: %d input cop%s of q, k, v, o, %d MiB per rank, rotated per step"
                   % (n_copies, "y" if n_copies == 1 else "ies", footprint // 2**20))},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                     "kernel": "attn_tcp_kernel", "kernel_ms": kern_ms, "kernel_ms_source": kern_src,
                     "kernel_ms_single_replay": kern_single,
                     "algorithmic_flops_per_launch": per_rank_flops,
                     "peak_source": f"bf16_tflops (burst) of {peak_kind} peaks"},
        "plan_build_ms": t_plan,
        "with_plan_build": None if ms_plan_step is None else {
            "value": job_flops / (ms_plan_step * 1e-3) / 1e12,
            "ms_per_step": ms_plan_step, "what": plan_how},
        "weak": weak,
        "e2e": {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "block_sparse_attention(q, k, v, mask) from pinned host buffers (plan built inside each "
                        "call); per step H2D of q, k, v, mask (+perms) and D2H of o, pipelined on copy streams"},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        "sustained": sustained,
    }
    if backward is not None:
        line["backward"] = backward
    if gpu_comparator is not None:
        ours_ms = ms_step
        if "ms_per_step" in gpu_comparator:
            gpu_comparator["this_library_speedup"] = gpu_comparator["ms_per_step"] / ours_ms
        line["gpu_comparator"] = gpu_comparator
    if per_config is not None:
        line["per_config"] = per_config
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
        line["cpu_dense_masked"] = cpu_dense_masked(wl, args.cpu_seconds)
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="headline")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="under torchrun: split the workload's (b,h) units over the ranks (strong) or give every "
                         "rank a copy (weak)")
    ap.add_argument("--sustained-seconds", type=float, default=2.0,
                    help="continuous load before the second (sustained) timing; 0 skips it")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    ap.add_argument("--ref-budget-s", type=float, default=90.0, help="total CPU time of the reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--no-backward", action="store_true", help="skip the backward-pass measurement")
    ap.add_argument("--no-gpu-comparator", action="store_true",
                    help="skip the torch.compile(flex_attention) comparator on the same GPU")
    ap.add_argument("--kernel", default="auto", help="kernel choice passed to block_sparse_attention")
    ap.add_argument("--configs", default=",".join(CONFIGS), help="configurations of the per-config object")
    ap.add_argument("--ncu-csv", default=None, help="ncu raw CSV of the same command: roofline traffic from it")
    ap.add_argument("--units", type=int, default=0,
                    help="time only the first U (b,h) units of the workload (a smaller case for ncu captures)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
