"""The device OCP MX e4m3 quantiser (hgemm_quantize_mx_e4m3) against the oracle's host
quantiser: bit-exact e4m3 bytes and e8m0 scale bytes (compared in the blocked layout the
MX GEMM reads, built from the oracle's row-major scales by the host converter), fp32 and
bf16 inputs, ragged shapes, special values; then quantise -> MX GEMM end to end."""
import numpy as np
import pytest
import torch

import oracle
from tests.gemm_cases import c_bits

pytestmark = pytest.mark.gpu


def _check(x32: np.ndarray, xdev: torch.Tensor):
    import hipgemm_b200 as hg
    q_ref, sf_ref = oracle.quantize_mx(x32)
    q, sf = hg.quantize_mx_e4m3(xdev)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sf.cpu().numpy(), hg.mx_sf_to_blocked(torch.from_numpy(sf_ref), x32.shape[1]).numpy())


@pytest.mark.parametrize("rows,K", [(1, 32), (3, 96), (128, 128), (300, 1056), (1000, 4128), (4096, 8192)])
def test_fp32_bit_exact(cuda_device, rows, K):
    rng = np.random.default_rng(rows * 7 + K)
    mag = np.ldexp(1.0, rng.integers(-20, 21, (rows, K // 32))).repeat(32, axis=1)
    x = (oracle.normal_f32(rows * K, seed=rows + K).reshape(rows, K) * mag).astype(np.float32)
    _check(x, torch.from_numpy(x).cuda())


@pytest.mark.parametrize("rows,K", [(2, 64), (257, 800), (2048, 4096)])
def test_bf16_bit_exact(cuda_device, rows, K):
    x = torch.from_numpy(oracle.normal_f32(rows * K, seed=3 * rows, mean=-0.5, stddev=4.0).reshape(rows, K))
    xb = x.to(torch.bfloat16)
    _check(xb.float().numpy(), xb.cuda())  # bf16 -> fp32 is exact


def test_special_values(cuda_device):
    """Zero, subnormal-only, infinite, NaN-containing, saturating and extreme-binade blocks."""
    K = 32 * 10
    x = np.zeros((3, K), dtype=np.float32)
    x[0, 32:64] = 1e-40                                   # subnormal amax: X clamps to -127
    x[0, 64:96] = np.linspace(-3e38, 3e38, 32)            # top binade: X = 127 - 8 = 119
    x[0, 96:128] = np.float32(np.inf)
    x[0, 100] = -np.inf
    x[0, 128:160] = np.linspace(-2, 2, 32)
    x[0, 130] = np.nan                                    # NaN ignored for amax, stays NaN
    x[0, 160:192] = np.ldexp(1.0, -126) * np.arange(32)   # smallest normals
    x[0, 192:224] = 448.0 * np.ldexp(1.0, np.arange(32) % 4)  # values above 448 * 2^X round/saturate
    x[1] = np.ldexp(1.0, -(np.arange(K) % 150)).astype(np.float32)  # down to 2^-149
    x[2] = -x[1]
    _check(x, torch.from_numpy(x).cuda())


def test_quantise_then_mx_gemm(cuda_device):
    import hipgemm_b200 as hg
    from tests.test_mx_gpu import _abs_products, _mismatches
    M, N, K = 512, 768, 2048
    xa = oracle.normal_f32(M * K, seed=5).reshape(M, K)
    xb = oracle.normal_f32(N * K, seed=6, stddev=0.05).reshape(N, K)
    qa, sfa = hg.quantize_mx_e4m3(torch.from_numpy(xa).cuda())
    qb, sfb = hg.quantize_mx_e4m3(torch.from_numpy(xb).cuda())
    c = hg.fp8_gemm_tn_mx(qa, qb, sfa, sfb)
    torch.cuda.synchronize()
    A, SFA = oracle.quantize_mx(xa)
    B, SFB = oracle.quantize_mx(xb)
    ref = oracle.gemm_mx(A, B, SFA, SFB)
    bad, info = _mismatches(c_bits(c), ref, _abs_products(A, B, SFA, SFB, np.arange(M), 1.0))
    assert bad == 0, info
    # MX keeps the product close to the fp32 one (per-block scales, e4m3 mantissas).
    exact = xa.astype(np.float64) @ xb.astype(np.float64).T
    got = oracle.bf16_to_f32(c_bits(c)).astype(np.float64)
    assert np.linalg.norm(got - exact) / np.linalg.norm(exact) < 0.05
