"""ctypes binding of the C ABI declared in ``include/linearard_b200.h``.

This is the reference-side binding a maintainer would add: plain pointers,
sizes and a ``cudaStream_t``.  The library is loaded from the package's
``_lib/`` directory; a missing library is an error (there is no fallback).
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "liblinearard_b200.so")

__all__ = ["LKLProblem", "LKLStrides", "LKLGroupItem", "lib", "check", "LKLError",
           "LKL_F16", "LKL_BF16", "MASK_DTYPES", "STATUS"]

LKL_F16, LKL_BF16 = 0, 1
LKL_MASK_BOOL, LKL_MASK_U8, LKL_MASK_I32, LKL_MASK_I64 = 0, 1, 2, 3
STATUS = {
    0: "LKL_OK", 1: "LKL_ERR_NULL_POINTER", 2: "LKL_ERR_BAD_SHAPE", 3: "LKL_ERR_BAD_HEAD_DIM",
    4: "LKL_ERR_BAD_DTYPE", 5: "LKL_ERR_MISALIGNED", 6: "LKL_ERR_WORKSPACE", 7: "LKL_ERR_LAUNCH",
    8: "LKL_ERR_NO_DEVICE", 9: "LKL_ERR_DEVICE_TIMEOUT", 10: "LKL_ERR_BAD_ALIAS",
    11: "LKL_ERR_TOO_LARGE", 12: "LKL_ERR_UNSUPPORTED",
}
MASK_DTYPES = {"bool": LKL_MASK_BOOL, "uint8": LKL_MASK_U8, "int32": LKL_MASK_I32,
               "int64": LKL_MASK_I64}

# every symbol the header declares
EXPORTS = ("lkl_abi_version", "lkl_status_string", "lkl_workspace_size", "lkl_lse",
           "lkl_kl_forward", "lkl_forward", "lkl_backward", "lkl_device_status",
           "lkl_last_path", "lkl_set_force_generic", "lkl_forward_noalloc",
           "lkl_last_cuda_error", "lkl_backward_workspace_size", "lkl_forward_strided",
           "lkl_backward_strided", "lkl_grouped_workspace_size", "lkl_forward_grouped",
           "lkl_backward_grouped", "lkl_backward_plan", "lkl_forward_workspace_size",
           "lkl_selftest_bounded_wait")


class LKLProblem(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int32), ("Hq", ctypes.c_int32), ("Hkv_s", ctypes.c_int32),
        ("Hkv_t", ctypes.c_int32), ("T", ctypes.c_int32), ("Ds", ctypes.c_int32),
        ("Dt", ctypes.c_int32), ("dtype_s", ctypes.c_int32), ("dtype_t", ctypes.c_int32),
        ("causal", ctypes.c_int32), ("mask_dtype", ctypes.c_int32),
        ("sm_scale_s", ctypes.c_float), ("sm_scale_t", ctypes.c_float),
    ]


class LKLStrides(ctypes.Structure):
    """Element strides (b, h, t) of a [B, H, T, D] input whose d stride is 1."""
    _fields_ = [("b", ctypes.c_int64), ("h", ctypes.c_int64), ("t", ctypes.c_int64)]


class LKLGroupItem(ctypes.Structure):
    """One (relation, layer) item of a grouped call (struct lkl_group_item)."""
    _fields_ = [("qs", ctypes.c_void_p), ("ks", ctypes.c_void_p), ("qt", ctypes.c_void_p),
                ("kt", ctypes.c_void_p), ("Hq", ctypes.c_int32), ("Hkv_s", ctypes.c_int32),
                ("Hkv_t", ctypes.c_int32), ("strided", ctypes.c_int32),
                ("lse_s", ctypes.c_void_p), ("lse_t", ctypes.c_void_p),
                ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p),
                ("strides", LKLStrides * 4)]


class LKLError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = _lib_handle.lkl_status_string(status).decode() if _lib_handle else ""
        if status == 7 and _lib_handle is not None:
            msg += f"; cudaError {_lib_handle.lkl_last_cuda_error()}"
        super().__init__(f"{where}: {STATUS.get(status, status)} ({msg})")


_lib_handle = None
_lock = threading.Lock()

_vp, _sz, _i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32
_P = ctypes.POINTER(LKLProblem)


def _declare(L):
    L.lkl_abi_version.restype = _i32
    L.lkl_status_string.restype = ctypes.c_char_p
    L.lkl_status_string.argtypes = [_i32]
    L.lkl_workspace_size.restype = _sz
    L.lkl_workspace_size.argtypes = [_P, _i32]
    L.lkl_forward_workspace_size.restype = _sz
    L.lkl_forward_workspace_size.argtypes = [_P, _i32]
    L.lkl_backward_workspace_size.restype = _sz
    L.lkl_backward_workspace_size.argtypes = [_P, _i32]
    L.lkl_lse.restype = _i32
    L.lkl_lse.argtypes = [_vp, _vp, _vp, _P, _vp, _vp, _sz, _vp]
    L.lkl_kl_forward.restype = _i32
    L.lkl_kl_forward.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _P, _vp, _vp, _sz, _vp]
    L.lkl_forward.restype = _i32
    L.lkl_forward.argtypes = [_vp, _vp, _vp, _vp, _vp, _P, _vp, _vp, _vp, _vp, _sz, _vp]
    L.lkl_backward.restype = _i32
    L.lkl_backward.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _P, _vp, _vp, _vp, _vp, _sz, _vp]
    L.lkl_device_status.restype = _i32
    L.lkl_selftest_bounded_wait.restype = _i32
    L.lkl_selftest_bounded_wait.argtypes = [ctypes.c_uint32, _vp]
    L.lkl_last_path.restype = _i32
    L.lkl_last_cuda_error.restype = _i32
    L.lkl_set_force_generic.restype = None
    L.lkl_set_force_generic.argtypes = [_i32]
    _S = ctypes.POINTER(LKLStrides)
    L.lkl_forward_strided.restype = _i32
    L.lkl_forward_strided.argtypes = [_vp, _vp, _vp, _vp, _S, _vp, _P, _vp, _vp, _vp, _vp, _sz,
                                      _vp]
    L.lkl_backward_strided.restype = _i32
    L.lkl_backward_strided.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _S, _vp, _P, _vp, _vp, _vp,
                                       _vp, _sz, _vp]
    _G = ctypes.POINTER(LKLGroupItem)
    L.lkl_grouped_workspace_size.restype = _sz
    L.lkl_grouped_workspace_size.argtypes = [_i32, _G, _P, _i32, _i32]
    L.lkl_forward_grouped.restype = _i32
    L.lkl_forward_grouped.argtypes = [_i32, _G, _vp, _P, _vp, _vp, _sz, _vp]
    L.lkl_backward_grouped.restype = _i32
    L.lkl_backward_grouped.argtypes = [_i32, _G, _vp, _P, _vp, _vp, _sz, _vp]
    L.lkl_backward_plan.restype = _i32
    L.lkl_backward_plan.argtypes = [_P, _i32, _sz, _i32, ctypes.POINTER(ctypes.c_int32)]
    L.lkl_forward_noalloc.restype = _i32
    L.lkl_forward_noalloc.argtypes = [_vp, _vp, _vp, _vp, _vp, _P, _vp, _vp, _vp, _vp]


def lib(path: str | None = None):
    """The loaded library (loaded once per process)."""
    global _lib_handle
    if _lib_handle is not None:
        return _lib_handle
    with _lock:
        if _lib_handle is None:
            p = path or os.environ.get("LINEARARD_B200_LIB", LIB_PATH)
            if not os.path.exists(p):
                raise RuntimeError(
                    f"liblinearard_b200.so not found at {p}; build it with "
                    "`python -m linearard_b200.build` (there is no CPU or Python fallback)")
            L = ctypes.CDLL(p)
            _declare(L)
            _lib_handle = L
    return _lib_handle


def check(status: int, where: str) -> None:
    if status != 0:
        raise LKLError(status, where)
