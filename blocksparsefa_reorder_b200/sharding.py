"""Multi-GPU partitioning: independent (b, h) units spread over ranks.

Every (b, h) pair of the forward is independent (the mask may differ per
(b, h); the permutation applies per token), so the work shards into
contiguous ranges of the flattened ``b * H + h`` index with no collective on
the hot path.  One process per GPU (``torchrun``); each rank runs the
single-GPU kernel on its own units.  Where a caller wants the full output on
one rank, :func:`gather_units` collects the shards with point-to-point
sends over the process group (NCCL over NVLink on B200, gloo on CPU).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist


def partition_units(num_units: int, world_size: int, weights: Optional[Sequence[float]] = None) -> list:
    """Split ``range(num_units)`` into ``world_size`` contiguous ``(lo, hi)``
    ranges.  Without weights the sizes differ by at most one; with per-unit
    weights (e.g. kept blocks per (b, h)) rank r's range ends at the last unit
    whose cumulative weight is within ``(r + 1) / world_size`` of the total,
    and the last rank takes the rest."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if num_units < 0:
        raise ValueError("num_units must be non-negative")
    if weights is None:
        base, extra = divmod(num_units, world_size)
        out, lo = [], 0
        for r in range(world_size):
            hi = lo + base + (1 if r < extra else 0)
            out.append((lo, hi))
            lo = hi
        return out
    if len(weights) != num_units:
        raise ValueError("one weight per unit")
    if any(w < 0 for w in weights):
        raise ValueError("weights must be non-negative")
    total = float(sum(weights))
    cum, acc = [], 0.0
    for w in weights:
        acc += float(w)
        cum.append(acc)
    out, lo = [], 0
    for r in range(world_size):
        if r == world_size - 1:
            hi = num_units
        else:
            target = total * (r + 1) / world_size
            hi = lo
            while hi < num_units and cum[hi] <= target + 1e-9 * max(1.0, total):
                hi += 1
        out.append((lo, hi))
        lo = hi
    return out


def local_heads(H: int, rank: int, world_size: int) -> tuple:
    """Head range ``[h0, h1)`` of this rank when heads are sharded (B = 1)."""
    return partition_units(H, world_size)[rank]


def split_parts(ranges: Sequence[tuple], parts: int) -> list:
    """Cut every rank's unit range into ``parts`` consecutive pieces (some
    empty when a rank has fewer units than parts), so that a rank can compute
    and ship its units piece by piece.  Returns one ``(pieces, offsets)`` per
    part: ``pieces[r] = (a, b)`` indexes rank r's local units, ``offsets[r]``
    is the global index of the piece's first unit (``gather_units``'s
    ``ranges`` / ``offsets`` for that part).  Every rank derives the same
    list, so all take the same collective steps."""
    if parts <= 0:
        raise ValueError("parts must be positive")
    out = []
    for i in range(parts):
        pieces, offsets = [], []
        for lo, hi in ranges:
            u = hi - lo
            a, b = u * i // parts, u * (i + 1) // parts
            pieces.append((a, b))
            offsets.append(lo + a)
        out.append((pieces, offsets))
    return out


def _global_rank(group, r: int) -> int:
    """Global rank of rank ``r`` of ``group`` (point-to-point calls take global ranks)."""
    return r if group is None else dist.get_global_rank(group, r)


def gather_units(local: torch.Tensor, ranges: Sequence[tuple], dst: int = 0, group=None, async_op: bool = False,
                 out: Optional[torch.Tensor] = None, offsets: Optional[Sequence[int]] = None):
    """Collect per-rank shards ``[hi - lo, ...]`` (rank r of ``group`` holds
    units ``ranges[r]``) into one ``[total, ...]`` tensor on group rank
    ``dst``; other ranks get ``None``.  The receives are posted together
    (``batch_isend_irecv``), so the shards arrive concurrently.  ``out`` /
    ``offsets`` (on ``dst``): receive rank r's shard into
    ``out[offsets[r]:offsets[r] + size]`` instead of a new tensor laid out by
    ``ranges``.  With ``async_op`` the call returns ``(full_or_None, works)``
    without waiting; wait on every work before reading the result (or reusing
    ``local``)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if len(ranges) != world:
        raise ValueError("one range per rank")
    lo, hi = ranges[rank]
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank}: local shard has {local.shape[0]} units, expected {hi - lo}")
    if offsets is None:
        offsets = [r[0] for r in ranges]
    elif len(offsets) != world:
        raise ValueError("one offset per rank")
    full, ops = None, []
    if rank == dst:
        if out is None:
            total = max(o + (b - a) for o, (a, b) in zip(offsets, ranges))
            out = torch.empty((total,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        full = out
        if hi > lo:
            full[offsets[rank]:offsets[rank] + hi - lo].copy_(local)
        for r in range(world):
            rlo, rhi = ranges[r]
            if r != dst and rhi > rlo:
                ops.append(dist.P2POp(dist.irecv, full[offsets[r]:offsets[r] + rhi - rlo], _global_rank(group, r),
                                      group))
    elif hi > lo:
        ops.append(dist.P2POp(dist.isend, local.contiguous(), _global_rank(group, dst), group))
    works = dist.batch_isend_irecv(ops) if ops else []
    if async_op:
        return full, works
    for w in works:
        w.wait()
    return full
