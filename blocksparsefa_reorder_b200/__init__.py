"""B200-native (sm_100a) block-sparse attention forward with token reordering.

Public API
----------
block_sparse_attention(q, k, v, block_mask, *, q_perm=None, kv_perm=None, ...)
    the forward: q, k, v ``[B, H, N, D]`` + BLOCK x BLOCK block mask (+ token
    permutations) in, output in original token order out.
BlockSparsePlan(block_mask, block)
    the per-tile list of kept key blocks, built on the GPU, reusable.
block_sparse_attention_backward(q, k, v, o, lse, dout, *, plan, plan_t, ...)
    gradients dq, dk, dv (BLOCK 64 / 128, bf16 / fp16, D 64 / 128; beyond the
    reference, which has no backward); block_sparse_attention_autograd wraps
    forward and backward as a differentiable op.
kernels.attn_fwd_block_sparse / attn_fwd_block_sparse_perm
    drop-ins for the reference's two Triton launches.
utils
    the reference's preprocessing surface (mask from coordinates, permutation
    files, update_idx_perm, apply_reordering, reverse_reordering) on the GPU.
runners.run_experiments_B200
    the reference runners' timing surface.
sharding
    (b, h) partitioning across GPUs and gathering of outputs.

The CUDA kernels live in ``_lib/libbsattn_b200.so`` (built by
``python -m blocksparsefa_reorder_b200.build``) behind the C ABI of
``include/bsattn_b200.h``.
"""

from ._lib import BsaError
from .api import (BlockSparsePlan, block_sparse_attention, block_sparse_attention_autograd,
                  block_sparse_attention_backward, infer_block, inverse_permutation, permute_rows, transposed_plan)

__all__ = ["BsaError", "BlockSparsePlan", "block_sparse_attention", "block_sparse_attention_autograd",
           "block_sparse_attention_backward", "infer_block", "inverse_permutation", "permute_rows",
           "transposed_plan"]
__version__ = "0.1.0"
