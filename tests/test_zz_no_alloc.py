"""The allocation-free plan build, bsa_build_plan_noalloc, called through the C ABI.

Some host programs never let a library allocate device memory: they hand out
every buffer from their own pool, or cannot afford the synchronisation an
allocation implies.  For them the library keeps the plan build's per-tile
scratch in a fixed device array instead of asking for a workspace.  This
test checks that variant against the ordinary bsa_build_plan on two calls in
a row (different masks, so stale scratch contents from the first call would
show up in the second) and that a mask with more tiles than the fixed array
holds is rejected.  The comparison is exact: the plan is integer data.

The file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import _lib

pytestmark = pytest.mark.gpu


def _mask(nb, slices, p, seed, dev):
    rng = np.random.default_rng(seed)
    m = rng.random((slices[0], slices[1], nb, nb)) < p
    return torch.from_numpy(m.astype(np.uint8)).to(dev)


def _plan_with_workspace(L, m, block, stream):
    mb, mh, nb = (int(x) for x in m.shape[:3])
    ptr_len, cap, ws = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_size_t()
    _lib.check(L.bsa_plan_sizes(mb, mh, nb, block, ctypes.byref(ptr_len), ctypes.byref(cap), ctypes.byref(ws)),
               "bsa_plan_sizes")
    tp = torch.empty(ptr_len.value, dtype=torch.int32, device=m.device)
    tc = torch.full((cap.value,), -1, dtype=torch.int32, device=m.device)
    work = torch.empty(max(1, ws.value // 4), dtype=torch.int32, device=m.device)
    _lib.check(L.bsa_build_plan(m.data_ptr(), m.stride(0), m.stride(1), m.stride(2), mb, mh, nb, block,
                                tp.data_ptr(), tc.data_ptr(), None, work.data_ptr(), ws.value, stream),
               "bsa_build_plan")
    return tp, tc


def _plan_noalloc(L, m, block, stream):
    mb, mh, nb = (int(x) for x in m.shape[:3])
    ptr_len, cap, ws = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_size_t()
    _lib.check(L.bsa_plan_sizes(mb, mh, nb, block, ctypes.byref(ptr_len), ctypes.byref(cap), ctypes.byref(ws)),
               "bsa_plan_sizes")
    tp = torch.empty(ptr_len.value, dtype=torch.int32, device=m.device)
    tc = torch.full((cap.value,), -1, dtype=torch.int32, device=m.device)
    _lib.check(L.bsa_build_plan_noalloc(m.data_ptr(), m.stride(0), m.stride(1), m.stride(2), mb, mh, nb, block,
                                        tp.data_ptr(), tc.data_ptr(), stream), "bsa_build_plan_noalloc")
    return tp, tc


@pytest.mark.parametrize("block", [128, 64])
def test_noalloc_plan_matches_workspace_plan_twice(dev, block):
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    # two calls in a row with different masks and tile counts
    cases = [(_mask(33, (2, 3), 0.3, 1, dev), "first"), (_mask(17, (1, 2), 0.6, 2, dev), "second")]
    for m, which in cases:
        ref_ptr, ref_col = _plan_with_workspace(L, m, block, stream)
        got_ptr, got_col = _plan_noalloc(L, m, block, stream)
        torch.cuda.synchronize()
        n = int(ref_ptr[-1].item())
        assert torch.equal(got_ptr, ref_ptr), which
        assert torch.equal(got_col[:n], ref_col[:n]), which


def test_noalloc_rejects_oversize_mask(dev):
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    dummy = torch.zeros(16, dtype=torch.int32, device=dev)
    nb = _lib.PLAN_NOALLOC_MAX_TILES + 1  # one tile per block row at BLOCK 128: one tile too many
    rc = L.bsa_build_plan_noalloc(dummy.data_ptr(), 0, 0, 0, 1, 1, nb, 128, dummy.data_ptr(), dummy.data_ptr(),
                                  stream)
    assert rc == 9  # BSA_ERR_WORKSPACE: more tiles than the fixed scratch holds
    torch.cuda.synchronize()
