"""Process pool running the oracle's port of the reference block loop on all
host cores (test / benchmark infrastructure only).

The reference's kernel is one program per query block
(``triton_kernels/BlockSparse_Naive.py:68-125``); the CPU baseline runs the
float32 numpy port of that program (:func:`oracle.attention._query_block`)
for many query blocks in parallel, one worker process per host core
(started with ``spawn``; q, k, v shared through ``multiprocessing``
shared memory; BLAS limited to one thread per worker).
"""

from __future__ import annotations

import math
import multiprocessing as mp
import os
import time
from multiprocessing import shared_memory

import numpy as np

from .attention import LOG2E, _query_block

_STATE = {}


def _init(names, shape, mask2d, block, qk_scale, p_dtype):
    arrs = []
    shms = []
    for nm in names:
        shm = shared_memory.SharedMemory(name=nm)
        shms.append(shm)
        arrs.append(np.ndarray(shape, dtype=np.float32, buffer=shm.buf))
    _STATE.update(q=arrs[0], k=arrs[1], v=arrs[2], shms=shms, mask=mask2d, block=block, qk_scale=qk_scale,
                  p_dtype=p_dtype)


def _run(mbs):
    s = _STATE
    acc = 0.0
    n = s["q"].shape[0]
    for mb in mbs:
        kept = np.nonzero(s["mask"][mb])[0]
        r0, r1 = mb * s["block"], min(n, (mb + 1) * s["block"])
        o, m = _query_block(s["q"][r0:r1], s["k"], s["v"], kept, s["block"], s["qk_scale"], s["p_dtype"])
        acc += float(o[0, 0])
    return acc


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class BlockLoopPool:
    """One head's q, k, v ([N, D] float32) and its [nb, nb] mask, with a pool
    of ``workers`` spawned processes that run query blocks on demand."""

    def __init__(self, q, k, v, mask2d, block: int, p_dtype=None, sm_scale=None, workers: int | None = None):
        q = np.ascontiguousarray(q, dtype=np.float32)
        self.shape = q.shape
        self.mask = np.asarray(mask2d, dtype=bool)
        self.block = block
        self.D = q.shape[1]
        self.workers = workers or host_cores()
        scale = 1.0 / math.sqrt(self.D) if sm_scale is None else sm_scale
        self._shms = []
        for a in (q, k, v):
            a = np.ascontiguousarray(a, dtype=np.float32)
            shm = shared_memory.SharedMemory(create=True, size=a.nbytes)
            np.ndarray(a.shape, dtype=np.float32, buffer=shm.buf)[...] = a
            self._shms.append(shm)
        old = {k2: os.environ.get(k2) for k2 in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS")}
        for k2 in old:
            os.environ[k2] = "1"
        try:
            ctx = mp.get_context("spawn")
            self.pool = ctx.Pool(self.workers, initializer=_init,
                                 initargs=([s.name for s in self._shms], self.shape, self.mask, block,
                                           np.float32(scale * LOG2E), p_dtype))
        finally:
            for k2, v2 in old.items():
                if v2 is None:
                    os.environ.pop(k2, None)
                else:
                    os.environ[k2] = v2
        # workers are up (bounded: a worker that cannot start must not hang the caller)
        self.pool.map_async(_run, [[] for _ in range(self.workers)]).get(timeout=300)

    def flops(self, query_blocks) -> float:
        kept = int(sum(int(self.mask[mb].sum()) for mb in query_blocks))
        return 4.0 * self.block * self.block * self.D * kept

    def run(self, query_blocks, timeout: float = 600.0) -> float:
        """Run the given query blocks across the pool; returns wall seconds."""
        qb = list(query_blocks)
        chunks = [qb[i::self.workers] for i in range(self.workers)]
        chunks = [c for c in chunks if c]
        t0 = time.perf_counter()
        self.pool.map_async(_run, chunks, chunksize=1).get(timeout=timeout)
        return time.perf_counter() - t0

    def close(self):
        self.pool.terminate()
        self.pool.join()
        for s in self._shms:
            s.close()
            s.unlink()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False
