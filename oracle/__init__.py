"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Restates nirw4nna/hipgemm's CPU GEMM (test.cpp:19-30), validator (test.cpp:32-47) and
input generator (utils.hpp:27-33), pinned bit for bit to the reference's own copies of
those functions compiled from its sources (oracle/reference.py; see oracle.h).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use it, and only as
the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_LIB: ctypes.CDLL | None = None
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_SIG = {
    "oracle_fp8_encode": (ctypes.c_uint8, [_f]),
    "oracle_fp8_decode": (_f, [ctypes.c_uint8]),
    "oracle_fp8_encode_array": (None, [_vp, ctypes.c_size_t, _vp]),
    "oracle_bf16_rne_array": (None, [_vp, ctypes.c_size_t, _vp]),
    "oracle_bf16_rne": (ctypes.c_uint16, [_f]),
    "oracle_bf16_to_float": (_f, [ctypes.c_uint16]),
    "oracle_normal_f32": (None, [_vp, ctypes.c_size_t, ctypes.c_uint64, _f, _f]),
    "oracle_init_random_fp8": (None, [_vp, ctypes.c_size_t, ctypes.c_uint64, _f, _f]),
    "oracle_quantize_e4m3": (_f, [_vp, ctypes.c_size_t, _vp]),
    "oracle_quantize_e4m3_with_scale": (_f, [_vp, ctypes.c_size_t, _f, _vp]),
    "oracle_make_quantized": (_f, [_vp, ctypes.c_size_t, ctypes.c_uint64, _f, _f]),
    "oracle_gemm_rows": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _i, _i]),
    "oracle_gemm_naive_rows": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _i, _i]),
    "oracle_gemm": (None, [_vp, _vp, _vp, _i, _i, _i, _f, _f, _i]),
    "oracle_gemm_row_list": (None, [_vp, _vp, _vp, _i, _i, _f, _f, _vp, _i, _i]),
    "oracle_validate": (ctypes.c_int64, [_vp, _vp, ctypes.c_int64, _f, _f, ctypes.POINTER(ctypes.c_int64)]),
    "oracle_validate_reference": (_i, [_vp, _vp, _i, _i]),
    "oracle_max_threads": (_i, []),
    "oracle_mt19937_nth": (ctypes.c_uint32, [ctypes.c_uint32, ctypes.c_uint64]),
    "oracle_quantize_mx_e4m3": (None, [_vp, _i, _i, _vp, _vp]),
    "oracle_gemm_mx_rows": (None, [_vp, _vp, _vp, _vp, _vp, _i, _i, _f, _f, _i, _i, _i]),
}

RTOL = 1e-2  # benchmark-config tolerance: |c - ref| <= RTOL*|ref| + ATOL per element
ATOL = 1e-3


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            build()
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIG.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def fp8_encode(x: float) -> int:
    return int(lib().oracle_fp8_encode(float(x)))


def fp8_decode(b: int) -> float:
    return float(lib().oracle_fp8_decode(int(b)))


def fp8_encode_array(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().oracle_fp8_encode_array(_p(x), x.size, _p(out))
    return out


def bf16_rne_array(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_bf16_rne_array(_p(x), x.size, _p(out))
    return out


def decode_table() -> np.ndarray:
    return np.array([fp8_decode(b) for b in range(256)], dtype=np.float32)


def bf16_rne(x: float) -> int:
    return int(lib().oracle_bf16_rne(float(x)))


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_f32(n: int, seed: int, mean: float = 0.0, stddev: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_normal_f32(_p(out), n, seed, mean, stddev)
    return out


def init_random_fp8(n: int, seed: int = 0, mean: float = -1.0, stddev: float = 1.0) -> np.ndarray:
    """utils.hpp:27-33 (reference defaults: seed 0, N(-1, 1), no scale)."""
    out = np.empty(n, dtype=np.uint8)
    lib().oracle_init_random_fp8(_p(out), n, seed, mean, stddev)
    return out


def quantize(x: np.ndarray) -> tuple[np.ndarray, float]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.shape, dtype=np.uint8)
    s = lib().oracle_quantize_e4m3(_p(x), x.size, _p(q))
    return q, float(s)


def quantize_with_scale(x: np.ndarray, scale: float) -> tuple[np.ndarray, float]:
    """Delayed scaling: (e4m3(x / scale), amax|x|)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.shape, dtype=np.uint8)
    amax = lib().oracle_quantize_e4m3_with_scale(_p(x), x.size, float(scale), _p(q))
    return q, float(amax)


def make_quantized(shape: tuple[int, int], seed: int, mean: float = 0.0, stddev: float = 1.0) -> tuple[np.ndarray, float]:
    q = np.empty(shape, dtype=np.uint8)
    s = lib().oracle_make_quantized(_p(q), q.size, seed, mean, stddev)
    return q, float(s)


def gemm(A: np.ndarray, B: np.ndarray, scale_a: float = 1.0, scale_b: float = 1.0, nthreads: int = 0) -> np.ndarray:
    """bf16 bits (uint16) of bf16(scale_a*scale_b * A . B^T), A: MxK, B: NxK e4m3 bytes."""
    M, K = A.shape
    N = B.shape[0]
    C = np.empty((M, N), dtype=np.uint16)
    lib().oracle_gemm(_p(A), _p(B), _p(C), M, N, K, scale_a, scale_b, nthreads)
    return C


def gemm_naive_rows(A, B, row_begin, row_end, scale_a=1.0, scale_b=1.0, nthreads=0) -> np.ndarray:
    """The reference loop nest (test.cpp:19-30) on rows [row_begin, row_end) (the timed baseline)."""
    M, K = A.shape
    N = B.shape[0]
    C = np.empty((row_end - row_begin, N), dtype=np.uint16)
    lib().oracle_gemm_naive_rows(_p(A), _p(B), _p(C), M, N, K, scale_a, scale_b, row_begin, row_end, nthreads)
    return C


def gemm_rows(A: np.ndarray, B: np.ndarray, rows, scale_a: float = 1.0, scale_b: float = 1.0,
              nthreads: int = 0) -> np.ndarray:
    """bf16 bits of the chosen rows of the product (len(rows) x N)."""
    rows = np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
    N, K = B.shape
    C = np.empty((rows.size, N), dtype=np.uint16)
    lib().oracle_gemm_row_list(_p(A), _p(B), _p(C), N, K, scale_a, scale_b, _p(rows), rows.size, nthreads)
    return C


def validate(C: np.ndarray, C_ref: np.ndarray, rtol: float = RTOL, atol: float = ATOL) -> tuple[int, int]:
    """(mismatch count, first bad flat index or -1) under |c-ref| <= rtol*|ref| + atol."""
    C = np.ascontiguousarray(C, dtype=np.uint16)
    C_ref = np.ascontiguousarray(C_ref, dtype=np.uint16)
    assert C.shape == C_ref.shape
    first = ctypes.c_int64(-1)
    bad = lib().oracle_validate(_p(C), _p(C_ref), C.size, rtol, atol, ctypes.byref(first))
    return int(bad), int(first.value)


def validate_reference(C: np.ndarray, C_ref: np.ndarray) -> bool:
    """test.cpp:32-47 as written (signed threshold, stops at the first mismatch)."""
    C = np.ascontiguousarray(C, dtype=np.uint16)
    C_ref = np.ascontiguousarray(C_ref, dtype=np.uint16)
    M, N = C.shape
    return bool(lib().oracle_validate_reference(_p(C), _p(C_ref), M, N))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def mt19937_nth(seed: int, n: int) -> int:
    """The n-th (1-based) output of std::mt19937(seed)."""
    return int(lib().oracle_mt19937_nth(seed, n))


def quantize_mx(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """OCP MX e4m3: (q rows x K, e8m0 scales rows x K/32) of a rows x K fp32 array."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    q = np.empty((rows, K), dtype=np.uint8)
    sf = np.empty((rows, K // 32), dtype=np.uint8)
    lib().oracle_quantize_mx_e4m3(_p(x), rows, K, _p(q), _p(sf))
    return q, sf


def gemm_mx(A, B, SFA, SFB, scale_a=1.0, scale_b=1.0, row_begin=0, row_end=None, nthreads=0) -> np.ndarray:
    """bf16 bits of rows [row_begin, row_end) of the block-scaled product."""
    M, K = A.shape
    N = B.shape[0]
    row_end = M if row_end is None else row_end
    C = np.empty((row_end - row_begin, N), dtype=np.uint16)
    lib().oracle_gemm_mx_rows(_p(A), _p(B), _p(np.ascontiguousarray(SFA)), _p(np.ascontiguousarray(SFB)), _p(C), N, K,
                              scale_a, scale_b, row_begin, row_end, nthreads)
    return C
