"""Multi-rank logic on CPU with the gloo backend (world size 2).

The GPU path shards (b, h) units across ranks with no collective; here each
rank computes its units with the CPU oracle (standing in for the GPU kernel,
which these CPU ranks cannot run) and rank 0 gathers the shards with
gather_units.  A failure test makes one rank raise before the gather and
checks that the other rank's receive ends with an error within the process
group's timeout instead of hanging."""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blocksparsefa_reorder_b200 import sharding
from oracle import attention as OA


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _worker_shard(rank, world, port, out_dir):
    try:
        _init(rank, world, port)
        B, H, N, D, block = 1, 4, 256, 32, 64
        g = np.random.default_rng(0)
        q, k, v = (g.standard_normal((B, H, N, D)).astype(np.float32) for _ in range(3))
        mask = g.random((1, 1, N // block, N // block)) < 0.5
        ranges = sharding.partition_units(B * H, world)
        lo, hi = ranges[rank]
        o, _ = OA.block_sparse_online(q, k, v, mask, block, heads=list(range(lo, hi)))
        local = torch.from_numpy(o.reshape(B * H, N, D)[lo:hi].copy())
        full = sharding.gather_units(local, ranges, dst=0)
        if rank == 0:
            ref, _ = OA.block_sparse_online(q, k, v, mask, block)
            np.save(os.path.join(out_dir, "err.npy"), np.array([np.abs(full.numpy() - ref.reshape(B * H, N, D)).max()]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"fail{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def test_sharded_units_gather_to_rank0(tmp_path):
    port = _free_port()
    mp.start_processes(_worker_shard, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    err = np.load(tmp_path / "err.npy")[0]
    assert err == 0.0


def _worker_subgroup(rank, world, port, out_dir):
    """World of 3; ranks 1 and 2 form a subgroup and gather to the
    subgroup's rank 0 (global rank 1): group ranks must be mapped to global
    ranks for the point-to-point calls.  The second gather places the shards
    at given offsets of a caller's tensor."""
    try:
        _init(rank, world, port)
        sub = dist.new_group([1, 2])
        if rank in (1, 2):
            ranges = [(0, 2), (2, 5)]
            grank = dist.get_rank(sub)
            lo, hi = ranges[grank]
            local = torch.arange(lo * 3, hi * 3, dtype=torch.float32).reshape(hi - lo, 3)
            full, works = sharding.gather_units(local, ranges, dst=0, group=sub, async_op=True)
            for w in works:
                w.wait()
            out = torch.zeros(7, 3) if grank == 0 else None
            placed = sharding.gather_units(local, ranges, dst=0, group=sub, out=out, offsets=[5, 0])
            if grank == 0:
                ref = torch.arange(15, dtype=torch.float32).reshape(5, 3)
                ok = torch.equal(full, ref) and torch.equal(placed[5:7], ref[0:2]) and torch.equal(placed[0:3],
                                                                                                   ref[2:5])
                with open(os.path.join(out_dir, "sub.txt"), "w") as f:
                    f.write("ok" if ok else "mismatch")
            else:
                assert full is None and placed is None
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"fail{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def test_gather_over_subgroup(tmp_path):
    port = _free_port()
    mp.start_processes(_worker_subgroup, args=(3, port, str(tmp_path)), nprocs=3, join=True, start_method="spawn")
    assert (tmp_path / "sub.txt").read_text() == "ok"


def _worker_parts(rank, world, port, out_dir):
    """The long-context step's gather: each rank ships its units in 4 parts
    (rank 0 has fewer units than parts, so some of its pieces are empty), all
    parts posted before any is waited on; rank 0 must end with every unit at
    its global index."""
    try:
        _init(rank, world, port)
        ranges = [(0, 3), (3, 8)]
        lo, hi = ranges[rank]
        local = torch.arange(lo * 2, hi * 2, dtype=torch.float32).reshape(hi - lo, 2)
        full = torch.full((8, 2), -1.0) if rank == 0 else None
        works = []
        for pieces, offsets in sharding.split_parts(ranges, 4):
            a, b = pieces[rank]
            _, w = sharding.gather_units(local[a:b], pieces, dst=0, async_op=True, out=full, offsets=offsets)
            works += w
        for w in works:
            w.wait()
        if rank == 0:
            ok = torch.equal(full, torch.arange(16, dtype=torch.float32).reshape(8, 2))
            with open(os.path.join(out_dir, "parts.txt"), "w") as f:
                f.write("ok" if ok else "mismatch")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"fail{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def test_gather_in_parts(tmp_path):
    assert sharding.split_parts([(0, 3), (3, 8)], 4) == [
        ([(0, 0), (0, 1)], [0, 3]), ([(0, 1), (1, 2)], [0, 4]), ([(1, 2), (2, 3)], [1, 5]),
        ([(2, 3), (3, 5)], [2, 6])]
    port = _free_port()
    mp.start_processes(_worker_parts, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "parts.txt").read_text() == "ok"


def _worker_fail(rank, world, port, out_dir):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # a rank that fails between steps, before its send
        os._exit(3)
    buf = torch.zeros(4)
    try:
        dist.recv(buf, src=1)
        ok = "received"
    except Exception as e:  # the peer is gone: the receive must fail, not hang
        ok = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(ok)
    os._exit(0)


def test_rank_failure_is_detected_not_hung(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker_fail, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung after its peer died"
    assert (tmp_path / "rank0.txt").read_text().startswith("error")
