"""ctypes binding of the C ABI in ``include/bsattn_b200.h``.

The shared library is built in-tree by ``blocksparsefa_reorder_b200.build``
into ``_lib/libbsattn_b200.so``.  Loading fails loudly when it is missing:
there is no CPU or library fallback for any entry point.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libbsattn_b200.so"

OK = 0
STATUS_NAMES = {
    0: "BSA_OK", 1: "BSA_ERR_INVALID_ARG", 2: "BSA_ERR_SHAPE", 3: "BSA_ERR_DTYPE", 4: "BSA_ERR_ALIGNMENT",
    5: "BSA_ERR_UNSUPPORTED", 6: "BSA_ERR_NOT_PERMUTATION", 7: "BSA_ERR_TIMEOUT", 8: "BSA_ERR_CUDA",
    9: "BSA_ERR_WORKSPACE", 10: "BSA_ERR_DEVICE",
}
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
INDEX_I32, INDEX_I64 = 0, 1
KERNEL_AUTO, KERNEL_SIMT, KERNEL_TCGEN05 = 0, 1, 2
DEVERR_TIMEOUT, DEVERR_PERM_RANGE, DEVERR_PERM_DUP, DEVERR_COORD, DEVERR_PLAN, DEVERR_ALIGN = 1, 2, 4, 8, 16, 32
ABI_VERSION = 2
PLAN_NOALLOC_MAX_TILES = 1 << 20


class Tensor4d(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64),
                ("stride_n", ctypes.c_int64)]


class Plan(ctypes.Structure):
    _fields_ = [("tile_ptr", ctypes.c_void_p), ("tile_col", ctypes.c_void_p), ("mask_b", ctypes.c_int32),
                ("mask_h", ctypes.c_int32), ("nb", ctypes.c_int32), ("block", ctypes.c_int32),
                ("tile_order", ctypes.c_void_p)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("N", ctypes.c_int32), ("D", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("q", Tensor4d), ("k", Tensor4d), ("v", Tensor4d), ("o", Tensor4d),
                ("sm_scale", ctypes.c_float), ("lse", ctypes.c_void_p), ("plan", Plan),
                ("err_flag", ctypes.c_void_p), ("kernel", ctypes.c_int32)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("N", ctypes.c_int32), ("D", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("q", Tensor4d), ("k", Tensor4d), ("v", Tensor4d), ("o", Tensor4d),
                ("dout", Tensor4d), ("dq", Tensor4d), ("dk", Tensor4d), ("dv", Tensor4d),
                ("sm_scale", ctypes.c_float), ("lse", ctypes.c_void_p), ("delta", ctypes.c_void_p),
                ("plan", Plan), ("plan_t", Plan), ("err_flag", ctypes.c_void_p)]


class BsaError(RuntimeError):
    """A C-ABI call returned a non-zero bsa_status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)} ({status_string(status)})")


_i32, _i64, _vp, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
PROTOS = {
    "bsa_abi_version": ([], ctypes.c_int),
    "bsa_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "bsa_device_supported": ([ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "bsa_plan_sizes": ([_i32, _i32, _i32, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_sz)],
                       ctypes.c_int),
    "bsa_build_plan": ([_vp, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp], ctypes.c_int),
    "bsa_build_plan_noalloc": ([_vp, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp], ctypes.c_int),
    "bsa_build_tile_order": ([_vp, _i32, _i32, _i32, _i32, _vp, _vp], ctypes.c_int),
    "bsa_fwd": ([ctypes.POINTER(FwdArgs), _vp], ctypes.c_int),
    "bsa_permute_rows": ([Tensor4d, Tensor4d, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _vp, _vp],
                         ctypes.c_int),
    "bsa_inverse_permutation": ([_vp, _i32, _i64, _vp, _vp, _vp], ctypes.c_int),
    "bsa_remap_indices": ([_vp, _i64, _vp, _i64, _vp, _vp, _vp], ctypes.c_int),
    "bsa_blockmask_from_coords": ([_vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "bsa_fwd_reordered_workspace_bytes": ([ctypes.POINTER(FwdArgs), ctypes.POINTER(_sz)], ctypes.c_int),
    "bsa_fwd_reordered": ([ctypes.POINTER(FwdArgs), _vp, _vp, _i32, _vp, _sz, _vp], ctypes.c_int),
    "bsa_test_arm_wait_timeout": ([ctypes.c_uint32], ctypes.c_int),
    "bsa_bwd": ([ctypes.POINTER(BwdArgs), _vp], ctypes.c_int),
}
EXPORTED = tuple(PROTOS)

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"{LIB_PATH} is missing: build the CUDA extension first "
                                       "(python -m blocksparsefa_reorder_b200.build)")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (argtypes, restype) in PROTOS.items():
                    fn = getattr(handle, name)
                    fn.argtypes = argtypes
                    fn.restype = restype
                if handle.bsa_abi_version() != ABI_VERSION:
                    raise RuntimeError(f"{LIB_PATH}: ABI version {handle.bsa_abi_version()} != {ABI_VERSION}")
                _lib = handle
    return _lib


def status_string(status: int) -> str:
    try:
        return lib().bsa_status_string(int(status)).decode()
    except Exception:
        return STATUS_NAMES.get(status, "unknown")


def check(status: int, what: str) -> None:
    if status != OK:
        raise BsaError(status, what)
