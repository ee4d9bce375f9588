"""ctypes binding of oracle/_ref/libref_cpu.so — TEST INFRASTRUCTURE ONLY.

The library is the reference's own CPU code: gemm_cpu and validate_matrix (test.cpp:19-47)
and init_random (utils.hpp:27-33), compiled from the reference's files where they lie by
`make -C oracle ref`, with the ROCm element types they use (fp8_4wave.hpp:15-16:
__hip_fp8_e4m3, __hip_bfloat16) restated in oracle/ref_shim_types.h.  It pins the oracle
(liboracle.so) to the reference: the tests compare the two bit for bit, and
tests/golden/reference/make_reference_golden.py records its outputs as fixtures for machines without
the reference's sources.  bench.py times its gemm_cpu as the reference's CPU baseline.

The library is built only where the reference's sources are present; once built it is an
ordinary file of the working tree and goes wherever the tree goes.  `available()` is False
where it is neither built nor buildable.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libref_cpu.so")
REFERENCE_DIR = os.environ.get("REFERENCE_DIR", "/root/reference")

_LIB: ctypes.CDLL | None = None
_vp = ctypes.c_void_p
_i = ctypes.c_int
_SIG = {
    "ref_gemm_cpu": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "ref_validate_matrix": (_i, [_vp, _vp, _i, _i]),
    "ref_init_random": (None, [_vp, ctypes.c_size_t, ctypes.c_size_t]),
    "ref_max_threads": (_i, []),
    "ref_set_num_threads": (None, [_i]),
    "ref_shim_e4m3_encode_array": (None, [_vp, ctypes.c_size_t, _vp]),
    "ref_shim_bf16_array": (None, [_vp, ctypes.c_size_t, _vp]),
}


def build() -> bool:
    """Builds the library if the reference's sources are here; True if it exists afterwards."""
    if os.path.isfile(os.path.join(REFERENCE_DIR, "test.cpp")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REFERENCE_DIR={REFERENCE_DIR}"], check=True)
    return os.path.isfile(LIB_PATH)


def available() -> bool:
    return os.path.isfile(LIB_PATH) or build()


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is not built and the reference's sources are absent")
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


def gemm_cpu(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """test.cpp:19-30: bf16 bits of A . B^T (A: M x K, B: N x K e4m3 bytes), unscaled, all threads."""
    A = np.ascontiguousarray(A, dtype=np.uint8)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    (M, K), N = A.shape, B.shape[0]
    assert B.shape[1] == K and M * K < 2**31 and N * K < 2**31 and M * N < 2**31  # the reference indexes in int
    C = np.empty((M, N), dtype=np.uint16)
    lib().ref_gemm_cpu(_p(A), _p(B), _p(C), M, N, K)
    return C


def validate_matrix(C: np.ndarray, C_ref: np.ndarray) -> bool:
    """test.cpp:32-47 as written (signed threshold; prints and stops at the first mismatch)."""
    C = np.ascontiguousarray(C, dtype=np.uint16)
    C_ref = np.ascontiguousarray(C_ref, dtype=np.uint16)
    assert C.shape == C_ref.shape
    M, N = C.shape
    return bool(lib().ref_validate_matrix(_p(C), _p(C_ref), M, N))


def init_random(n: int, seed: int = 0) -> np.ndarray:
    """utils.hpp:27-33: n e4m3 bytes from std::mt19937(seed) and normal_distribution<float>(-1, 1)."""
    out = np.empty(n, dtype=np.uint8)
    lib().ref_init_random(_p(out), n, seed)
    return out


def max_threads() -> int:
    return int(lib().ref_max_threads())


def set_num_threads(n: int) -> None:
    """OpenMP threads for this thread's next gemm_cpu calls."""
    lib().ref_set_num_threads(int(n))


def shim_e4m3_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().ref_shim_e4m3_encode_array(_p(x), x.size, _p(out))
    return out


def shim_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ref_shim_bf16_array(_p(x), x.size, _p(out))
    return out
