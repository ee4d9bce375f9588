"""Generates the committed golden fixtures for the FP8 TN GEMM (tests/golden/*.npz).

    python tests/golden/make_golden.py

The reference ships no golden vectors and its CPU path (test.cpp:19-30) cannot be
built here (it needs ROCm headers), so the expected outputs are computed by a third,
deliberately plain restatement written only in this file: e4m3 decoded from the OCP
FP8 definition with exact rational arithmetic, products formed exactly, the k-sum
accumulated one term at a time in IEEE fp32 (numpy.float32 scalars, as test.cpp:23-26
does), the scale applied as (scale_a*scale_b)*acc in fp32 and the result rounded to
bf16 with round-to-nearest-even by integer bit manipulation.  Inputs come from the
reference's generator (mt19937 + normal_distribution<float>, utils.hpp:27-33) through
the C++ oracle, which is the only part of the oracle this script uses.

Each fixture holds A (M x K e4m3 bytes), B (N x K e4m3 bytes), scale_a, scale_b and C
(M x N bf16 bits).  The tests check the oracle bit-for-bit and the GPU kernel within
|d| <= 1e-2*|ref| + 1e-3 against them.
"""
from __future__ import annotations

import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

# (name, M, N, K, seed_a, seed_b, mean_a, std_a, mean_b, std_b, scaled)
CASES = [
    ("tiny_scaled", 4, 8, 32, 0, 1, 0.0, 1.0, 0.0, 1.0, True),
    ("ragged_scaled", 17, 24, 48, 3, 4, 0.0, 1.0, 0.0, 1.0, True),
    ("ffn_like_scaled", 9, 16, 160, 5, 6, 0.0, 1.0, 0.0, 0.02, True),
    ("reference_mode", 16, 16, 128, 0, 0, -1.0, 1.0, -1.0, 1.0, False),  # test.cpp:70-71 seeds, N(-1,1), unscaled
    ("long_k_scaled", 3, 8, 1024, 7, 8, 0.0, 1.0, 0.0, 1.0, True),
]


def e4m3_value(b: int) -> Fraction | None:
    """OCP FP8 E4M3: S.EEEE.MMM, bias 7, S.1111.111 = NaN, no infinities."""
    sign = -1 if b & 0x80 else 1
    e = (b >> 3) & 0xF
    m = b & 0x7
    if e == 0xF and m == 0x7:
        return None
    if e == 0:
        return sign * Fraction(m, 8) * Fraction(1, 2 ** 6)
    return sign * (1 + Fraction(m, 8)) * (Fraction(2) ** (e - 7))


def bf16_bits_rne(x: np.float32) -> int:
    u = int(np.float32(x).view(np.uint32))
    if np.isnan(x):
        return ((u >> 16) & 0x8000) | 0x7FC0
    lsb = (u >> 16) & 1
    return ((u + 0x7FFF + lsb) >> 16) & 0xFFFF


def plain_gemm(A: np.ndarray, B: np.ndarray, sa: float, sb: float) -> np.ndarray:
    M, K = A.shape
    N = B.shape[0]
    table = [e4m3_value(b) for b in range(256)]
    s = np.float32(np.float32(sa) * np.float32(sb))
    C = np.empty((M, N), dtype=np.uint16)
    for i in range(M):
        for j in range(N):
            acc = np.float32(0.0)
            for k in range(K):
                prod = np.float32(float(table[A[i, k]] * table[B[j, k]]))  # exact in fp32
                acc = np.float32(acc + prod)
            C[i, j] = bf16_bits_rne(np.float32(s * acc))
    return C


def main() -> None:
    import oracle
    for (name, M, N, K, seed_a, seed_b, ma, sa_, mb, sb_, scaled) in CASES:
        if scaled:
            A, sa = oracle.make_quantized((M, K), seed_a, ma, sa_)
            B, sb = oracle.make_quantized((N, K), seed_b, mb, sb_)
        else:
            A = oracle.init_random_fp8(M * K, seed_a, ma, sa_).reshape(M, K)
            B = oracle.init_random_fp8(N * K, seed_b, mb, sb_).reshape(N, K)
            sa = sb = 1.0
        C = plain_gemm(A, B, sa, sb)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, A=A, B=B, scale_a=np.float32(sa), scale_b=np.float32(sb), C=C,
                            shape=np.array([M, N, K]))
        print(f"wrote {path}: {M}x{N}x{K} scaled={scaled}")


if __name__ == "__main__":
    main()
