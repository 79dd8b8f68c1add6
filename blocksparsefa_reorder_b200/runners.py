"""Experiment runners with the reference's call surface.

``run_experiments_B200(args, block_mask, seq_len, row_perm=None,
col_perm=None, device="cuda:0", dtype=torch.float16)`` mirrors the four
reference runners (e.g. ``BlockSparseTriton_Naive.py:10-18``): it draws
``q, k, v = randn([1, H, N, D])`` after ``torch.manual_seed(42)`` on
``device``, then times

* "with reordering": gather q by ``row_perm`` and k, v by ``col_perm``, the
  attention kernel, scatter o back (``BlockSparseTriton_Naive.py:129-161``);
* "without reordering": the attention kernel alone on pre-permuted inputs
  (``:209-225``),

after ``REPEATS_WARMUP`` warm-up calls, over ``REPEATS_TIMING`` calls, and
prints the reference's two lines (``Average time with reordering: X ms`` /
``Average time without reordering: X ms``).  Times are taken with CUDA
events on the current stream.  The reference names
``run_experiments_BSTriton_Naive`` / ``run_experiments_BSTriton_Fused`` map
to this runner.
"""

from __future__ import annotations

from typing import Optional

import torch

from .api import BlockSparsePlan, block_sparse_attention, infer_block, permute_rows

REPEATS_WARMUP = 10
REPEATS_TIMING = 25


def _time(fn, warmup: int, reps: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / reps


def run_experiments_B200(args, block_mask: torch.Tensor, seq_len: int, row_perm: Optional[torch.Tensor] = None,
                         col_perm: Optional[torch.Tensor] = None, device: str = "cuda:0",
                         dtype: torch.dtype = torch.float16, *, batch_size: int = 1, warmup: int = REPEATS_WARMUP,
                         reps: int = REPEATS_TIMING, verbose: bool = True) -> dict:
    torch.manual_seed(42)
    nheads, d = args.num_heads, args.head_dim
    q = torch.randn(batch_size, nheads, seq_len, d, device=device, dtype=dtype)
    k = torch.randn(batch_size, nheads, seq_len, d, device=device, dtype=dtype)
    v = torch.randn(batch_size, nheads, seq_len, d, device=device, dtype=dtype)
    mask = block_mask.to(device)
    block = infer_block(seq_len, int(mask.shape[-1]))
    plan = BlockSparsePlan(mask, block)
    rp = None if row_perm is None else row_perm.to(device)
    cp = None if col_perm is None else col_perm.to(device)

    def with_reordering():
        return block_sparse_attention(q, k, v, plan=plan, q_perm=rp, kv_perm=cp)

    t_with = _time(with_reordering, warmup, reps)
    qn = q if rp is None else permute_rows(q, rp, 2, inverse=False)
    kn = k if cp is None else permute_rows(k, cp, 2, inverse=False)
    vn = v if cp is None else permute_rows(v, cp, 2, inverse=False)
    o = torch.empty_like(q)

    def without_reordering():
        return block_sparse_attention(qn, kn, vn, plan=plan, out=o)

    t_without = _time(without_reordering, warmup, reps)
    if verbose:
        print(f"Average time with reordering: {t_with:.3f} ms")
        print(f"Average time without reordering: {t_without:.3f} ms")
    return {"ms_with_reordering": t_with, "ms_without_reordering": t_without}


run_experiments_BSTriton_Naive = run_experiments_B200
run_experiments_BSTriton_Fused = run_experiments_B200
