"""CPU oracle for the block-sparse attention path (test infrastructure only).

This package restates, on the CPU and in numpy, what the reference
(KutayTasci/BlockSparseFA_Reorder) computes on its hot path:

* ``oracle.preprocess`` -- token coordinates -> block mask, permutation
  inverse / remap / gather / scatter (reference ``utils.py:51-84, 236-288``),
  plus the per-tile CSR list of kept key blocks that the CUDA kernels consume
  (the ascending key-block scan of ``triton_kernels/BlockSparse_Naive.py:25-32``).
* ``oracle.attention`` -- the masked-softmax attention forward: a float64 dense
  definition (the parity checker) and a float32 port of the reference's
  online-softmax block loop (``triton_kernels/BlockSparse_Naive.py:5-125``),
  which also serves as the timed CPU baseline.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against golden vectors produced by the reference itself (its ``utils.py`` run
on CPU and its two Triton kernels run under ``TRITON_INTERPRET=1``), committed
under ``tests/golden/`` together with the script that made them.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and its ``--impl reference`` arm) may import this package,
and only as the checker / the CPU baseline.  The product package
``blocksparsefa_reorder_b200`` never imports it and has no CPU fallback.
"""

from . import attention, preprocess  # noqa: F401
