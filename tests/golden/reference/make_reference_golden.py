"""Generates tests/golden/reference/gemm_cpu.npz from the reference's own CPU code.

    make -C oracle ref && python tests/golden/reference/make_reference_golden.py

oracle/_ref/libref_cpu.so is the reference's gemm_cpu, validate_matrix (test.cpp:19-47) and
init_random (utils.hpp:27-33) compiled from its files (oracle/Makefile, target `ref`), with
the ROCm element types restated (oracle/ref_shim_types.h).  This script runs it on:

  test_cpp_256   the reference test's own flow (test.cpp:70-76) at M = N = K = 256: A and B
                 both from init_random with its default seed 0, C = gemm_cpu(A, B);
  test_cpp_ragged the same generator (A seed 1, B seed 2) at 100 x 72 x 320, sizes that are
                 not multiples of any tile;
  bytes_ragged   every finite e4m3 code (uniform bytes, NaN codes replaced), 37 x 40 x 384:
                 subnormals, +-448 and large products, which N(-1, 1) never reaches.
(N is a multiple of 8 in all three: the library's C ABI needs 16-byte rows of C.)

Each case stores A (M x K e4m3 bytes), B (N x K), C (M x N bf16 bits) and the reference
validator's verdict on C against itself (`self_valid`: False when C holds a negative value,
the signed-threshold behaviour of test.cpp:39).  The tests check the oracle bit for bit and
the GPU kernel within |d| <= 1e-2*|ref| + 1e-3 against these outputs, on machines without
the reference's sources too.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, ROOT)

OUT = os.path.join(HERE, "gemm_cpu.npz")


def cases():
    from oracle import reference as ref
    rng = np.random.default_rng(20240611)
    out = {}
    for name, M, N, K, sa, sb in (("test_cpp_256", 256, 256, 256, 0, 0), ("test_cpp_ragged", 100, 72, 320, 1, 2)):
        out[name] = (ref.init_random(M * K, sa).reshape(M, K), ref.init_random(N * K, sb).reshape(N, K))
    A = rng.integers(0, 256, (37, 384), dtype=np.uint8)
    B = rng.integers(0, 256, (40, 384), dtype=np.uint8)
    A[(A & 0x7F) == 0x7F] = 0x7E  # NaN codes -> 448
    B[(B & 0x7F) == 0x7F] = 0x01  # NaN codes -> the smallest subnormal
    out["bytes_ragged"] = (A, B)
    return out


def main() -> None:
    from oracle import reference as ref
    if not ref.available():
        sys.exit("the reference's CPU library is not built and its sources are absent")
    arrays = {}
    for name, (A, B) in cases().items():
        C = ref.gemm_cpu(A, B)
        arrays[f"{name}_A"] = A
        arrays[f"{name}_B"] = B
        arrays[f"{name}_C"] = C
        arrays[f"{name}_self_valid"] = np.array(ref.validate_matrix(C, C))
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes): {sorted(cases())}")


if __name__ == "__main__":
    main()
