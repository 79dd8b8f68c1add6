"""The bounded waits of the tcgen05 attention kernel, made to run out on the
GPU without a fault.

Every mbarrier wait in the kernel gives up after a time limit (2 s in
production), ORs BSA_DEVERR_TIMEOUT into the error word and raises the CTA's
abort flag, and every role then drains its TMA loads and MMAs, frees the
tensor memory and returns.  ``bsa_test_arm_wait_timeout`` arms the next
forward with a 1 ms limit and makes one softmax warp of CTA 0 withhold one
barrier arrival (nothing else is ever counted on that barrier), so that wait
runs out.  The host must see the timeout through ``check_errors``, and the
next forwards on the same stream must be correct: the CTA gave its
work-counter slot back and the context is intact.
"""

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import BlockSparsePlan, block_sparse_attention
from blocksparsefa_reorder_b200 import _lib
from oracle import attention as OA

pytestmark = pytest.mark.gpu

TOL_16 = 2e-2


@pytest.mark.parametrize("permuted", [False, True])
def test_wait_timeout_reported_then_next_forward_correct(dev, permuted):
    B, H, N, D, block = 1, 4, 2048, 128, 128
    nb = N // block
    rng = np.random.default_rng(11)
    mask = rng.random((1, 1, nb, nb)) < 0.4
    mask[..., np.arange(nb), np.arange(nb)] = True  # every tile has work, CTA 0's included
    g = torch.Generator(device="cpu").manual_seed(12)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    qp = torch.randperm(N, generator=g).to(dev) if permuted else None
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    good = block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kernel="tcgen05", check_errors=True)

    L = _lib.lib()
    assert L.bsa_test_arm_wait_timeout(1000) == 0
    with pytest.raises(RuntimeError, match="device wait timed out"):
        block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kernel="tcgen05", check_errors=True)

    # the context still works, and the launch after it is correct (and the one
    # that reuses the timed-out launch's work-counter slot, 64 launches later)
    for _ in range(65):
        o = block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kernel="tcgen05", check_errors=True)
        assert torch.equal(o, good)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref, _ = OA.reordered_attention(f(q), f(k), f(v), mask, block, None if qp is None else qp.cpu().numpy())
    assert np.abs(f(o) - ref).max() <= TOL_16
