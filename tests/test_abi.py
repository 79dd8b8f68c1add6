"""The C-ABI shared library loads, exports every symbol include/*.h declares,
and rejects invalid arguments on the host (no GPU work is issued)."""

import ctypes
import re
from pathlib import Path

import pytest

from blocksparsefa_reorder_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = []
    for h in (ROOT / "include").glob("*.h"):
        names += re.findall(r"BSA_API\s+[\w\s\*]+?\b(bsa_\w+)\s*\(", h.read_text())
    return sorted(set(names))


def test_library_loads_and_exports_all_declared_symbols():
    L = _lib.lib()
    declared = _declared()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(_lib.PROTOS)
    assert L.bsa_abi_version() == _lib.ABI_VERSION


def test_status_strings():
    L = _lib.lib()
    assert L.bsa_status_string(0) == b"ok"
    assert b"aligned" in L.bsa_status_string(4)
    assert L.bsa_status_string(999) == b"unknown status"


def test_plan_sizes():
    L = _lib.lib()
    ptr_len, cap, ws = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_size_t()
    assert L.bsa_plan_sizes(1, 16, 128, 128, ctypes.byref(ptr_len), ctypes.byref(cap), ctypes.byref(ws)) == 0
    assert (ptr_len.value, cap.value, ws.value) == (16 * 128 + 1, 16 * 128 * 128, 16 * 128 * 4)
    # BLOCK 64: a tile holds two block rows; odd nb rounds up
    assert L.bsa_plan_sizes(2, 1, 9, 64, ctypes.byref(ptr_len), ctypes.byref(cap), ctypes.byref(ws)) == 0
    assert ptr_len.value == 2 * 5 + 1 and cap.value == 2 * 5 * 9
    assert L.bsa_plan_sizes(1, 1, 8, 32, None, None, None) == 5       # unsupported BLOCK
    assert L.bsa_plan_sizes(0, 1, 8, 64, None, None, None) == 1       # invalid size


def _args(**kw):
    a = _lib.FwdArgs()
    a.B, a.H, a.N, a.D = kw.get("B", 1), kw.get("H", 2), kw.get("N", 256), kw.get("D", 64)
    a.dtype = kw.get("dtype", _lib.DTYPE_BF16)
    fake = 0x1000
    for t in ("q", "k", "v", "o"):
        setattr(a, t, _lib.Tensor4d(fake, 2 * 256 * 64, 256 * 64, 64))
    a.sm_scale = kw.get("scale", 0.125)
    a.plan = _lib.Plan(fake, fake, kw.get("mb", 1), kw.get("mh", 1), kw.get("nb", 2), kw.get("block", 128))
    a.kernel = kw.get("kernel", 0)
    return a


@pytest.mark.parametrize("kw,status", [
    ({"B": 0}, 1), ({"dtype": 7}, 3), ({"block": 32}, 5), ({"nb": 3}, 2), ({"mh": 3}, 2),
    ({"scale": -1.0}, 5), ({"scale": float("nan")}, 5), ({"kernel": 9}, 1),
])
def test_fwd_validation_on_host(kw, status):
    L = _lib.lib()
    a = _args(**kw)
    assert L.bsa_fwd(ctypes.byref(a), None) == status


def test_fwd_null_pointers_rejected():
    L = _lib.lib()
    a = _args()
    a.q = _lib.Tensor4d(None, 0, 0, 0)
    assert L.bsa_fwd(ctypes.byref(a), None) == 1
    assert L.bsa_fwd(None, None) == 1


def test_other_entry_points_validate_on_host():
    L = _lib.lib()
    t = _lib.Tensor4d(0x1000, 0, 0, 64)
    assert L.bsa_permute_rows(t, t, 1, 1, 8, 64, 2, 0x2000, 1, 0, None, None) == 1   # dst == src
    assert L.bsa_permute_rows(t, _lib.Tensor4d(0x3000, 0, 0, 64), 1, 1, 8, 64, 9, 0x2000, 1, 0, None, None) == 3
    assert L.bsa_inverse_permutation(None, 1, 0, None, None, None) == 0               # empty: nothing to do
    assert L.bsa_inverse_permutation(0x1000, 5, 4, 0x2000, None, None) == 3
    assert L.bsa_remap_indices(None, -1, None, 0, None, None, None) == 1
    assert L.bsa_build_tile_order(None, 1, 1, 4, 128, 0x1000, None) == 1               # no tile_ptr
    assert L.bsa_build_tile_order(0x1000, 1, 1, 4, 96, 0x2000, None) == 5              # block size
    assert L.bsa_blockmask_from_coords(None, None, 0, 0, 64, 1, 1, None, None, None, None, None) == 1
    assert L.bsa_test_arm_wait_timeout(10) == 1                                       # below 100 us: refused
    assert L.bsa_test_arm_wait_timeout(3_000_000) == 1                                # above 2 s: refused
    size = ctypes.c_size_t()
    assert L.bsa_fwd_reordered_workspace_bytes(ctypes.byref(_args()), ctypes.byref(size)) == 0
    # fused tcgen05 forward: k', v' of 1*2*256*64 bf16 each (Q and O go through the permutation in-kernel)
    assert size.value == 2 * 2 * 256 * 64 * 2
    assert L.bsa_fwd_reordered_workspace_bytes(ctypes.byref(_args(kernel=1)), ctypes.byref(size)) == 0
    # SIMT forward: q', k', v', o' (lse not requested)
    assert size.value == 4 * 2 * 256 * 64 * 2
    a = _args()
    assert L.bsa_fwd_reordered(ctypes.byref(a), None, 0x1000, 1, None, 0, None) == 9   # workspace missing
    assert L.bsa_fwd_reordered(ctypes.byref(_args(kernel=1)), 0x1000, None, 1, None, 0, None) == 9
    assert L.bsa_fwd_reordered(ctypes.byref(a), 0x1000, None, 7, 0x1000, 1 << 30, None) == 3  # perm dtype


def _bwd_args(**kw):
    a = _lib.BwdArgs()
    a.B, a.H, a.N, a.D = kw.get("B", 1), kw.get("H", 2), kw.get("N", 256), kw.get("D", 64)
    a.dtype = kw.get("dtype", _lib.DTYPE_BF16)
    fake = 0x1000
    for t in ("q", "k", "v", "o", "dout", "dq", "dk", "dv"):
        setattr(a, t, _lib.Tensor4d(fake, 2 * 256 * 64, 256 * 64, 64))
    a.sm_scale = kw.get("scale", 0.125)
    a.lse = kw.get("lse", fake)
    a.delta = kw.get("delta", fake)
    for pl in ("plan", "plan_t"):
        setattr(a, pl, _lib.Plan(fake, fake, 1, 1, kw.get("nb", 2), kw.get("block", 128)))
    return a


def test_bwd_rejects_invalid_arguments_on_the_host():
    L = _lib.lib()
    assert L.bsa_bwd(None, None) == 1
    assert L.bsa_bwd(ctypes.byref(_bwd_args(dtype=_lib.DTYPE_F32)), None) == 3   # f16 / bf16 only
    assert L.bsa_bwd(ctypes.byref(_bwd_args(D=96)), None) == 5                   # D 64 / 128 only
    assert L.bsa_bwd(ctypes.byref(_bwd_args(block=32, nb=8)), None) == 5         # BLOCK 64 / 128 only
    assert L.bsa_bwd(ctypes.byref(_bwd_args(nb=3)), None) == 2                   # nb vs N
    assert L.bsa_bwd(ctypes.byref(_bwd_args(lse=None)), None) == 1               # lse required
    assert L.bsa_bwd(ctypes.byref(_bwd_args(delta=None)), None) == 1             # delta workspace required
    assert L.bsa_bwd(ctypes.byref(_bwd_args(scale=-1.0)), None) == 5
    assert L.bsa_bwd(ctypes.byref(_bwd_args(delta=0x1004)), None) == 4           # delta not 16-byte aligned
