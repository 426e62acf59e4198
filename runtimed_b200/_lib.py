"""ctypes binding of libruntimed_b200.so (the C ABI declared in include/rtd.h).

The library is the product: there is no Python or CPU fallback.  Loading fails
loudly when the shared library is missing (build it with
``python -m runtimed_b200.build``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libruntimed_b200.so")

RTD_OK = 0
RTD_ERR_INVALID = 1
RTD_ERR_SHAPE = 2
RTD_ERR_UNSUPPORTED = 3
RTD_ERR_TRUNCATED = 4
RTD_ERR_CUDA = 5
RTD_ERR_OOM = 6
RTD_ERR_PEER_TIMEOUT = 7
RTD_ERR_INDEX = 8
RTD_ERR_DEVICE = 9
RTD_ERR_WORKSPACE = 10

TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 8, 12, 14
TYPE_INT4_MARLIN = 1001  # rtd_marlin_upload handles (not a GGUF type)
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
FP8_W8A16, FP8_W8A8 = 0, 1

# Every exported symbol with (restype, argtypes).
_c = ctypes
_vp = _c.c_void_p
_i64 = _c.c_int64
_u32 = _c.c_uint32
SIGNATURES = {
    "rtd_init": (_c.c_int32, [_c.c_int, _c.POINTER(_vp)]),
    "rtd_destroy": (_c.c_int32, [_vp]),
    "rtd_last_error": (_c.c_char_p, [_vp]),
    "rtd_kernel_launches": (_c.c_uint64, []),
    "rtd_check_device_status": (_c.c_int32, [_vp, _vp]),
    "rtd_block_geometry": (_c.c_int32, [_u32, _c.POINTER(_i64), _c.POINTER(_i64)]),
    "rtd_qweight_upload": (_c.c_int32, [_vp, _u32, _vp, _c.c_size_t, _i64, _i64, _c.POINTER(_vp)]),
    "rtd_qweight_free": (_c.c_int32, [_vp]),
    "rtd_marlin_upload": (_c.c_int32, [_vp, _vp, _vp, _i64, _i64, _c.POINTER(_vp)]),
    "rtd_qweight_to_device": (_c.c_int32, [_vp, _vp, _c.POINTER(_vp)]),
    "rtd_qweight_rows": (_c.c_int32, [_vp, _i64, _i64, _c.POINTER(_vp)]),
    "rtd_qweight_info": (_c.c_int32, [_vp, _c.POINTER(_u32), _c.POINTER(_i64), _c.POINTER(_i64),
                                      _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t)]),
    "rtd_qlinear": (_c.c_int32, [_vp, _vp, _vp, _u32, _i64, _i64, _vp, _vp, _u32, _i64, _vp]),
    "rtd_qlinear_noalloc": (_c.c_int32, [_vp, _vp, _u32, _i64, _i64, _vp, _vp, _u32, _i64, _vp]),
    "rtd_noalloc_check_status": (_c.c_int32, [_c.c_int, _vp]),
    "rtd_tp_comm_create": (_c.c_int32, [_vp, _c.c_int, _c.c_int, _i64, _vp, _vp]),
    "rtd_tp_comm_open": (_c.c_int32, [_vp, _vp]),
    "rtd_tp_comm_destroy": (_c.c_int32, [_vp]),
    "rtd_tp_qlinear_row": (_c.c_int32, [_vp, _vp, _vp, _u32, _i64, _i64, _vp, _vp, _u32, _i64, _vp]),
    "rtd_tp_allreduce": (_c.c_int32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _u32, _i64, _vp]),
    "rtd_rmsnorm": (_c.c_int32, [_vp, _vp, _i64, _vp, _u32, _i64, _vp, _c.c_float, _i64, _i64, _vp, _u32, _i64,
                                 _vp]),
    "rtd_rope_kv_append": (_c.c_int32, [_vp, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _c.c_int32, _c.c_int32,
                                        _c.c_int32, _c.c_int32, _c.c_float, _vp, _vp, _vp, _c.c_int32, _vp, _vp,
                                        _u32, _vp, _vp]),
    "rtd_attention_paged": (_c.c_int32, [_vp, _vp, _i64, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_float, _vp, _vp,
                                         _vp, _c.c_int32, _c.c_int32, _vp, _vp, _u32, _vp, _u32, _i64, _vp]),
    "rtd_silu_mul": (_c.c_int32, [_vp, _vp, _u32, _i64, _vp, _u32, _i64, _i64, _i64, _vp, _u32, _i64, _vp]),
    "rtd_argmax": (_c.c_int32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "rtd_qlinear_argmax": (_c.c_int32, [_vp, _vp, _vp, _u32, _i64, _i64, _vp, _vp, _u32, _i64, _vp, _vp]),
    "rtd_qlinear_argmax_keys": (_c.c_int32, [_vp, _vp, _vp, _u32, _i64, _i64, _vp, _i64, _vp, _vp]),
    "rtd_qembed": (_c.c_int32, [_vp, _vp, _vp, _i64, _vp, _vp]),
    "rtd_qdequant": (_c.c_int32, [_vp, _vp, _vp, _vp]),
    "rtd_fp8weight_upload": (_c.c_int32, [_vp, _vp, _vp, _i64, _i64, _i64, _c.POINTER(_vp)]),
    "rtd_fp8weight_free": (_c.c_int32, [_vp]),
    "rtd_fp8_linear": (_c.c_int32, [_vp, _vp, _vp, _u32, _i64, _i64, _vp, _u32, _i64, _u32, _vp]),
    "rtd_fp8_encode": (_c.c_int32, [_vp, _vp, _i64, _vp, _vp]),
}

_lib = None


class RtdError(RuntimeError):
    """A non-zero rtd_status; `.status` carries the code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"rtd status {status}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: the CUDA extension is not built "
                "(run `python -m runtimed_b200.build`); there is no fallback path")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, ctx=None) -> None:
    if status != RTD_OK:
        msg = lib().rtd_last_error(ctx)
        raise RtdError(status, msg.decode() if msg else "")
