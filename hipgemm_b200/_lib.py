"""ctypes binding of libhipgemm_b200.so (the C ABI declared in include/hipgemm_b200.h).

There is no fallback: if the library is missing the import of this module raises,
and every GPU entry point runs the sm_100a kernels or returns an error.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhipgemm_b200.so")

HGEMM_OK = 0
HGEMM_ERR_INVALID_VALUE = -1
HGEMM_ERR_ALIGNMENT = -2
HGEMM_ERR_UNSUPPORTED = -3
HGEMM_ERR_CUDA = -4
HGEMM_ERR_NO_DEVICE = -5
HGEMM_ERR_DEVICE_TIMEOUT = -6

HGEMM_SCHEDULE_AUTO = 0
HGEMM_SCHEDULE_DATA_PARALLEL = 1
HGEMM_SCHEDULE_STREAM_K = 2

HGEMM_DTYPE_F32 = 0
HGEMM_DTYPE_BF16 = 1


class HgemmError(RuntimeError):
    """A negative status code from the C ABI (never a silent fallback)."""

    def __init__(self, code: int, where: str = ""):
        self.code = code
        msg = lib().hgemm_error_string(code).decode() if _LIB is not None else str(code)
        super().__init__(f"{where}: hgemm status {code}: {msg}" if where else f"hgemm status {code}: {msg}")


_LIB: ctypes.CDLL | None = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_SIGNATURES = {
    "hgemm_fp8_tn": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp]),
    "hgemm_fp8_tn_rows": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "hgemm_fp8_tn_config": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i]),
    "hgemm_fp8_tn_ex": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp, ctypes.c_size_t]),
    "hgemm_workspace_bytes": (_i, [_i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_size_t)]),
    "hgemm_plan": (_i, [_i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_int)]),
    "hgemm_debug_schedule": (_i, [ctypes.c_longlong, _i, _i, _i, ctypes.POINTER(ctypes.c_int)]),
    "hgemm_debug_work_items": (_i, [_i, _i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_int), _i]),
    "hgemm_debug_split_work": (_i, [_i, _i, _i, _i, ctypes.POINTER(ctypes.c_int)]),
    "hgemm_debug_choose": (_i, [_i, _i, _i, _i, ctypes.POINTER(ctypes.c_int), _i]),
    "hgemm_fp8_tn_rows_allgather": (_i, [_vp, _vp, ctypes.POINTER(ctypes.c_void_p), _i, _i, _i, _i, _i, _i, _i,
                                        _vp, _vp, _vp]),
    "hgemm_ipc_export": (_i, [_vp, _vp, ctypes.POINTER(ctypes.c_size_t)]),
    "hgemm_ipc_import": (_i, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "hgemm_ipc_close": (_i, [_vp]),
    "hgemm_quantize_e4m3": (_i, [_vp, _i, ctypes.c_size_t, _vp, _vp, _vp]),
    "hgemm_fp8_tn_from_host": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "hgemm_fp8_tn_mx": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "hgemm_fp8_tn_mx_config": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "hgemm_mx_num_configs": (_i, []),
    "hgemm_debug_stalled_gemm": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "hgemm_quantize_mx_e4m3": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "hgemm_quantize_e4m3_delayed": (_i, [_vp, _i, ctypes.c_size_t, _vp, _vp, _vp, _vp]),
    "hgemm_mx_config_name": (ctypes.c_char_p, [_i]),
    "hgemm_mx_sf_bytes": (ctypes.c_size_t, [_i, _i]),
    "hgemm_host_mx_sf_to_blocked": (_i, [_vp, _i, _i, _vp]),
    "hgemm_num_configs": (_i, []),
    "hgemm_config_resident_ctas": (_i, [_i]),
    "hgemm_config_name": (ctypes.c_char_p, [_i]),
    "hgemm_device_status": (_i, [ctypes.POINTER(ctypes.c_uint32)]),
    "hgemm_debug_workspace_pool_created": (_i, [_i]),
    "hgemm_fp8_tn_static_scratch": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp]),
    "hgemm_error_string": (ctypes.c_char_p, [_i]),
    "hgemm_version": (ctypes.c_char_p, []),
    "hgemm_host_init_random": (None, [_vp, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]),
    "hgemm_host_make_quantized": (ctypes.c_float, [_vp, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_float,
                                                   ctypes.c_float]),
    "hgemm_host_quantize_e4m3": (ctypes.c_float, [_vp, ctypes.c_size_t, _vp]),
    "hgemm_host_fp8_encode": (ctypes.c_uint8, [ctypes.c_float]),
    "hgemm_host_bf16_rne": (ctypes.c_uint16, [ctypes.c_float]),
    "hgemm_host_fp8_encode_array": (None, [_vp, ctypes.c_size_t, _vp]),
}


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m hipgemm_b200.build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(code: int, where: str = "") -> None:
    if code != HGEMM_OK:
        raise HgemmError(code, where)


def config_names() -> list[str]:
    L = lib()
    return [L.hgemm_config_name(i).decode() for i in range(L.hgemm_num_configs())]
