"""The backward pass (dq, dk, dv) against float32 autograd of the dense masked
attention on the same inputs.

The reference has no backward (its kernels write the row LSE M,
``triton_kernels/BlockSparse_Naive.py:119-122``, and nothing consumes it), so
the checker is the definition: O = softmax(QK^T * scale, -inf outside the
kept blocks) V, rows with no kept block O = 0, differentiated by torch in
float32 from the bf16 / fp16 inputs.  Tolerance per gradient: max |ours -
ref| <= 1.5e-2 (bf16) or 3e-3 (fp16) times max |ref| (P and dS are rounded to
16 bits on the way into the tensor cores, as in the forward; measured 3-4.5e-3
for bf16 and 3-6e-4 for fp16 on these cases).
"""

import math

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import (BlockSparsePlan, block_sparse_attention, block_sparse_attention_autograd,
                                        block_sparse_attention_backward, transposed_plan)

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 1.5e-2, torch.float16: 3e-3}


def _mask(H, nb, seed):
    rng = np.random.default_rng(seed)
    m = rng.random((1, H, nb, nb)) < 0.35
    m[..., np.arange(nb), np.arange(nb)] = True
    m[0, 0, 2, :] = False        # a query block row that keeps nothing
    m[0, 1, :, nb - 2] = False   # a key block that no query block keeps
    return m


def _reference(q, k, v, mask, block, scale, dout):
    """float32 autograd of the dense masked attention (finite fill, so rows
    that keep nothing stay NaN-free; their output is set to 0)."""
    B, H, N, D = q.shape
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    tm = torch.from_numpy(mask).to(q.device)
    full = tm.repeat_interleave(block, -2).repeat_interleave(block, -1)[..., :N, :N].expand(B, H, N, N)
    s = (qf @ kf.transpose(-1, -2)) * scale
    s = s.masked_fill(~full, -1e30)
    p = torch.softmax(s, dim=-1)
    keep = full.any(-1, keepdim=True)
    o = torch.where(keep, p @ vf, torch.zeros((), device=q.device))
    o.backward(dout.float())
    return qf.grad, kf.grad, vf.grad


def _close(a, ref):
    return (a.float() - ref).abs().max().item() <= TOL[a.dtype] * ref.abs().max().item()


@pytest.mark.parametrize("block", [128, 64])
@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16), (128, torch.float16),
                                     (64, torch.bfloat16)])
def test_backward_matches_autograd(dev, D, dtype, block):
    """Per-head masks with a query block that keeps nothing and a key block
    no query block keeps, a partial last block; at BLOCK 64 the 128-row tiles
    (and 128-key tiles of the dK/dV kernel) hold blocks kept by one half only."""
    B, H = 1, 2
    N = 128 * 6 - 40  # a partial last block
    nb = (N + block - 1) // block
    mask = _mask(H, nb, seed=D)
    g = torch.Generator(device="cpu").manual_seed(D + 1)
    q, k, v, dout = (torch.randn(B, H, N, D, generator=g).to(dtype).to(dev) for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    plan_t = transposed_plan(plan, torch.from_numpy(mask).to(dev))
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    dq, dk, dv = block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=plan_t,
                                                 check_errors=True)
    rq, rk, rv = _reference(q, k, v, mask, block, scale, dout)
    assert torch.isfinite(dq.float()).all() and torch.isfinite(dk.float()).all() and torch.isfinite(dv.float()).all()
    assert _close(dq, rq), (dq.float() - rq).abs().max().item()
    assert _close(dk, rk), (dk.float() - rk).abs().max().item()
    assert _close(dv, rv), (dv.float() - rv).abs().max().item()
    # nothing kept -> exactly zero: the empty query block row's dq, the unkept key block's dk / dv
    assert torch.count_nonzero(dq[0, 0, 2 * block:3 * block]) == 0
    assert torch.count_nonzero(dk[0, 1, (nb - 2) * block:(nb - 1) * block]) == 0
    assert torch.count_nonzero(dv[0, 1, (nb - 2) * block:(nb - 1) * block]) == 0
    # deterministic: no atomics
    dq2, dk2, dv2 = block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=plan_t)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


def test_backward_many_tiles_and_broadcast_mask(dev):
    """A mask shared by every (b, h) (broadcast [1, 1, nb, nb]) over B 2 H 4,
    N 2048 (more tiles than one wave of CTAs)."""
    B, H, N, D, block = 2, 4, 2048, 128, 128
    nb = N // block
    rng = np.random.default_rng(5)
    mask = rng.random((1, 1, nb, nb)) < 0.2
    mask[..., np.arange(nb), np.arange(nb)] = True
    g = torch.Generator(device="cpu").manual_seed(6)
    q, k, v, dout = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(4))
    m = torch.from_numpy(mask).to(dev)
    plan = BlockSparsePlan(m, block)
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    dq, dk, dv = block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=transposed_plan(plan, m),
                                                 check_errors=True)
    rq, rk, rv = _reference(q, k, v, mask, block, 1.0 / math.sqrt(D), dout)
    assert _close(dq, rq) and _close(dk, rk) and _close(dv, rv)


def test_backward_block64_causal_fp16(dev):
    """The density sweep's kind of mask (fp16, BLOCK 64, causal with the
    diagonal kept, below-diagonal blocks at p = 0.3) over B 2 H 3."""
    B, H, N, D, block = 2, 3, 64 * 24, 128, 64
    nb = N // block
    rng = np.random.default_rng(12)
    mask = np.tril(rng.random((1, 1, nb, nb)) < 0.3)
    mask[..., np.arange(nb), np.arange(nb)] = True
    g = torch.Generator(device="cpu").manual_seed(13)
    q, k, v, dout = (torch.randn(B, H, N, D, generator=g).to(torch.float16).to(dev) for _ in range(4))
    m = torch.from_numpy(mask).to(dev)
    plan = BlockSparsePlan(m, block)
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    dq, dk, dv = block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=transposed_plan(plan, m),
                                                 check_errors=True)
    rq, rk, rv = _reference(q, k, v, mask, block, 1.0 / math.sqrt(D), dout)
    assert _close(dq, rq) and _close(dk, rk) and _close(dv, rv)


def test_autograd_wrapper(dev):
    B, H, N, D, block = 1, 2, 512, 64, 128
    nb = N // block
    mask = _mask(H, nb, seed=9)
    g = torch.Generator(device="cpu").manual_seed(10)
    q, k, v, dout = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(4))
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = block_sparse_attention_autograd(qa, ka, va, torch.from_numpy(mask).to(dev), block=block)
    o.backward(dout)
    m = torch.from_numpy(mask).to(dev)
    plan = BlockSparsePlan(m, block)
    o2, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    assert torch.equal(o.detach(), o2)
    dq, dk, dv = block_sparse_attention_backward(q, k, v, o2, lse, dout, plan=plan, plan_t=transposed_plan(plan, m))
    assert torch.equal(qa.grad, dq) and torch.equal(ka.grad, dk) and torch.equal(va.grad, dv)
