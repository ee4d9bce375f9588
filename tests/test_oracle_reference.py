"""The oracle pinned to the reference's own CPU code (no GPU).

oracle/_ref/libref_cpu.so is the reference's gemm_cpu, validate_matrix (test.cpp:19-47) and
init_random (utils.hpp:27-33) compiled from its files, with only the ROCm element types
restated (oracle/ref_shim_types.h).  Where it is built (or its sources are here to build it)
the oracle must reproduce it bit for bit; everywhere, the oracle must reproduce the fixtures
it generated (tests/golden/reference/gemm_cpu.npz).
"""
import os

import numpy as np
import pytest

import oracle
from oracle import reference as ref

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "reference", "gemm_cpu.npz")
CASES = ("test_cpp_256", "test_cpp_ragged", "bytes_ragged")

needs_ref = pytest.mark.skipif(not ref.available(), reason="the reference's CPU library is not built and "
                                                           "its sources are absent")


@pytest.fixture(scope="module")
def golden():
    return np.load(FIXTURE)


@pytest.mark.parametrize("case", CASES)
def test_oracle_reproduces_reference_fixture(golden, case):
    A, B, C = golden[f"{case}_A"], golden[f"{case}_B"], golden[f"{case}_C"]
    assert np.array_equal(oracle.gemm(A, B), C)
    assert np.array_equal(oracle.gemm_naive_rows(A, B, 0, A.shape[0]), C)
    assert oracle.validate(C, C) == (0, -1)
    assert oracle.validate_reference(C, C) == bool(golden[f"{case}_self_valid"])


def test_reference_fixture_inputs_are_the_reference_generator(golden):
    """test.cpp:70-71: both operands from init_random with the default seed 0."""
    A, B = golden["test_cpp_256_A"], golden["test_cpp_256_B"]
    assert np.array_equal(A.ravel(), oracle.init_random_fp8(A.size, 0))
    assert np.array_equal(B.ravel(), oracle.init_random_fp8(B.size, 0))
    assert np.array_equal(golden["test_cpp_ragged_A"].ravel(), oracle.init_random_fp8(100 * 320, 1))
    assert np.array_equal(golden["test_cpp_ragged_B"].ravel(), oracle.init_random_fp8(72 * 320, 2))


@needs_ref
@pytest.mark.parametrize("case", CASES)
def test_reference_library_reproduces_its_fixture(golden, case):
    A, B = golden[f"{case}_A"], golden[f"{case}_B"]
    assert np.array_equal(ref.gemm_cpu(A, B), golden[f"{case}_C"])


@needs_ref
@pytest.mark.parametrize("seed,n", [(0, 1), (0, 300001), (1, 4096), (7, 65537), (2**31 + 5, 1000)])
def test_init_random_matches_reference(seed, n):
    assert np.array_equal(ref.init_random(n, seed), oracle.init_random_fp8(n, seed))


@needs_ref
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (1, 64, 7), (64, 1, 129), (33, 17, 200), (128, 96, 512), (5, 3, 4096)])
@pytest.mark.parametrize("inputs", ["reference", "bytes"])
def test_gemm_matches_reference_loop(M, N, K, inputs):
    if inputs == "reference":
        A = ref.init_random(M * K, M).reshape(M, K)
        B = ref.init_random(N * K, N + 1).reshape(N, K)
    else:
        rng = np.random.default_rng(M * 1000 + N * 10 + K)
        A = rng.integers(0, 256, (M, K), dtype=np.uint8)
        B = rng.integers(0, 256, (N, K), dtype=np.uint8)
        A[(A & 0x7F) == 0x7F] = 0x3F
        B[(B & 0x7F) == 0x7F] = 0xC1
    C = ref.gemm_cpu(A, B)
    assert np.array_equal(oracle.gemm(A, B), C)
    assert np.array_equal(oracle.gemm_naive_rows(A, B, 0, M), C)
    rows = np.arange(M)[::3]
    assert np.array_equal(oracle.gemm_rows(A, B, rows), C[rows])


@needs_ref
def test_validate_matrix_matches_reference():
    rng = np.random.default_rng(3)
    pos = oracle.bf16_rne_array(rng.uniform(1.0, 100.0, (16, 24)).astype(np.float32))
    neg = oracle.bf16_rne_array(rng.uniform(-100.0, -1.0, (16, 24)).astype(np.float32))
    cases = [(pos, pos), (neg, neg)]
    off = pos.copy()
    off[5, 7] += 200  # far outside 1 %
    cases.append((off, pos))
    near = pos.copy()
    near[2, 3] += 1  # one bf16 ulp: inside 1 % of values >= 1
    cases.append((near, pos))
    nan = pos.copy()
    nan[0, 0] = 0x7FC0
    cases += [(nan, pos), (pos, nan)]
    for C, C_ref in cases:
        assert ref.validate_matrix(C, C_ref) == oracle.validate_reference(C, C_ref)
    assert ref.validate_matrix(pos, pos) and not ref.validate_matrix(neg, neg)


@needs_ref
def test_restated_rocm_conversions_agree_with_oracle():
    """The shim's e4m3 and bf16 conversions (restating ROCm 7.2.2's host conversions) against
    the oracle's, written separately: every e4m3 midpoint +-1 ulp, ties, saturation, signed
    zeros, subnormals, and a strided sweep of fp32 bit patterns."""
    table = oracle.decode_table()
    fin = np.sort(table[np.isfinite(table) & (table >= 0)])
    mids = ((fin[1:].astype(np.float64) + fin[:-1]) / 2).astype(np.float32)
    pts = np.concatenate([mids, np.nextafter(mids, np.float32(0)), np.nextafter(mids, np.float32(1e9)), fin,
                          np.array([448, 464, 465, 480, 1e6, np.inf, 0.0], dtype=np.float32)])
    pts = np.concatenate([pts, -pts])
    sweep = (np.arange(0, 2**32, 4099, dtype=np.uint64).astype(np.uint32)).view(np.float32)
    sweep = sweep[~np.isnan(sweep)]
    x = np.concatenate([pts, sweep])
    assert np.array_equal(ref.shim_e4m3_encode(x), oracle.fp8_encode_array(x))
    finite = x[np.isfinite(x)]
    assert np.array_equal(ref.shim_bf16(finite), oracle.bf16_rne_array(finite))


@needs_ref
def test_reference_test_at_its_default_size():
    """test.cpp:49-76 at its default MDIM = NDIM = KDIM = 4096 (test.cpp:6-16): A and B both
    init_random(seed 0), C_ref = gemm_cpu(A, B).  The oracle reproduces every bit, and the
    reference's validator accepts it."""
    n = 4096
    A = ref.init_random(n * n, 0).reshape(n, n)
    assert np.array_equal(A.ravel()[:1 << 20], oracle.init_random_fp8(1 << 20, 0))
    C_ref = ref.gemm_cpu(A, A)
    C = oracle.gemm(A, A)
    assert np.array_equal(C, C_ref)
    assert ref.validate_matrix(C, C_ref)
