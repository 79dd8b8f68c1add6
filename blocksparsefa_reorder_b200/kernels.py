"""Kernel-level drop-ins for the reference's two Triton launches.

The reference runners launch ``_attn_fwd_block_sparse[grid](...)``
(``triton_kernels/BlockSparse_Naive.py:69-77``, launched at
``BlockSparseTriton_Naive.py:142-156``) and
``_attn_fwd_block_sparse_perm[grid](...)``
(``triton_kernels/BlockSparse_Fused.py:116-127``, launched at
``BlockSparseTriton_Fused.py:95-111``).  These functions take the same
arguments by name, write ``o`` and ``M`` in place like those kernels, and run
the sm_100a kernels instead.  Launch-tuning arguments (``STAGE``,
``warp_specialize``, ``IS_HOPPER``, ``num_warps``, ``num_stages``) are
accepted and ignored.

Deliberate differences: any (B, H) works for the permuted variant (the
reference indexes its expanded ``[B,H,N,D]`` permutation views as
``[B,H,N]``, which is only right for ``B*H == 1``); bf16 and fp32 work besides
fp16; ``BLOCK_M == BLOCK_N`` must be 64 or 128.
"""

from __future__ import annotations

from .api import BlockSparsePlan, block_sparse_attention


def _check_blocks(BLOCK_M: int, BLOCK_N: int, N_CTX: int, block_mask) -> int:
    if BLOCK_M != BLOCK_N:
        raise ValueError("BLOCK_M must equal BLOCK_N (the mask has one block size)")
    if BLOCK_M not in (64, 128):
        raise ValueError("BLOCK_M must be 64 or 128")
    nb = (N_CTX + BLOCK_M - 1) // BLOCK_M
    if block_mask.shape[-1] != nb or block_mask.shape[-2] != nb:
        raise ValueError(f"block_mask must end in [{nb}, {nb}] for N_CTX={N_CTX}, BLOCK={BLOCK_M}")
    return BLOCK_M


def attn_fwd_block_sparse(sm_scale, M, Z, H, q, k, v, o, block_mask, N_CTX, HEAD_DIM, BLOCK_M, BLOCK_N, STAGE=1,
                          warp_specialize=False, IS_HOPPER=False, plan=None, **_launch):
    """``o, M = attention(q, k, v)`` over the kept blocks of ``block_mask``
    (``[Z, H, nb, nb]`` or broadcastable), written in place; ``M`` is the
    base-2 log-sum-exp per row (``BlockSparse_Naive.py:119-122``)."""
    block = _check_blocks(BLOCK_M, BLOCK_N, N_CTX, block_mask)
    if tuple(q.shape) != (Z, H, N_CTX, HEAD_DIM):
        raise ValueError("q shape does not match Z, H, N_CTX, HEAD_DIM")
    if plan is None:
        plan = BlockSparsePlan(block_mask, block)
    block_sparse_attention(q, k, v, plan=plan, sm_scale=sm_scale, return_lse=True, out=o, lse_out=M)
    return o, M


def attn_fwd_block_sparse_perm(sm_scale, M, Z, H, q, k, v, o, block_mask, N_CTX, q_perm, kv_perm, HEAD_DIM,
                               BLOCK_M, BLOCK_N, STAGE=1, warp_specialize=False, IS_HOPPER=False, plan=None,
                               **_launch):
    """The permuted variant (``BlockSparse_Fused.py:115-223``): q rows are read
    at ``q_perm``, k / v rows at ``kv_perm``, the mask is in the permuted
    order, and ``o`` / ``M`` are written at the ``q_perm`` rows, i.e. in the
    original order."""
    block = _check_blocks(BLOCK_M, BLOCK_N, N_CTX, block_mask)
    if tuple(q.shape) != (Z, H, N_CTX, HEAD_DIM):
        raise ValueError("q shape does not match Z, H, N_CTX, HEAD_DIM")
    if plan is None:
        plan = BlockSparsePlan(block_mask, block)
    block_sparse_attention(q, k, v, plan=plan, q_perm=q_perm, kv_perm=kv_perm, sm_scale=sm_scale,
                           return_lse=True, out=o, lse_out=M)
    return o, M
