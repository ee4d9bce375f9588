"""The device quantiser (hgemm_quantize_e4m3) against the oracle's host quantiser
(amax/448 scale, e4m3 of x / scale): bit-exact bytes and scale, fp32 and bf16 inputs,
ragged lengths, and end to end into the GEMM."""
import numpy as np
import pytest
import torch

import oracle
from tests.gemm_cases import c_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, 1_000_003, 4096 * 4096])
def test_fp32_bit_exact(cuda_device, n):
    import hipgemm_b200 as hg
    x = oracle.normal_f32(n, seed=n, mean=0.0, stddev=3.0)
    q_ref, s_ref = oracle.quantize(x)
    q, s = hg.quantize_e4m3(torch.from_numpy(x).cuda())
    assert float(s.item()) == s_ref
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("n", [8, 9, 4096 + 5, 2_000_000])
def test_bf16_bit_exact(cuda_device, n):
    import hipgemm_b200 as hg
    xb = torch.from_numpy(oracle.normal_f32(n, seed=7 * n, mean=-1.0, stddev=1.0)).to(torch.bfloat16)
    q_ref, s_ref = oracle.quantize(xb.float().numpy())  # bf16 -> fp32 is exact
    q, s = hg.quantize_e4m3(xb.cuda())
    assert float(s.item()) == s_ref
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_zero_tensor_and_empty(cuda_device):
    import hipgemm_b200 as hg
    q, s = hg.quantize_e4m3(torch.zeros(4097, device="cuda"))
    assert float(s.item()) == 1.0 and int(q.count_nonzero()) == 0
    q, s = hg.quantize_e4m3(torch.zeros(0, device="cuda"))
    assert float(s.item()) == 1.0 and q.numel() == 0


def test_quantise_then_gemm(cuda_device):
    """Quantise fp32 A and B on the GPU, multiply, compare with the oracle on the same bytes."""
    import hipgemm_b200 as hg
    M, N, K = 512, 768, 1024
    xa = torch.from_numpy(oracle.normal_f32(M * K, 1).reshape(M, K)).cuda()
    xb = torch.from_numpy(oracle.normal_f32(N * K, 2).reshape(N, K)).cuda()
    qa, sa = hg.quantize_e4m3(xa)
    qb, sb = hg.quantize_e4m3(xb)
    c = hg.fp8_gemm_tn(qa, qb, sa, sb)
    A = qa.cpu().numpy()
    B = qb.cpu().numpy()
    ref = oracle.gemm(A, B, float(sa.item()), float(sb.item()))
    assert oracle.validate(c_bits(c), ref)[0] == 0


@pytest.mark.parametrize("n", [1, 17, 4096 + 7, 3_000_001])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_delayed_scaling_bit_exact(cuda_device, n, dtype):
    """One-pass delayed scaling: bytes and amax equal the oracle's for a carried-over scale."""
    import hipgemm_b200 as hg
    x = oracle.normal_f32(n, seed=n + 1, mean=0.25, stddev=2.0)
    xt = torch.from_numpy(x)
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
        x = xt.float().numpy()
    scale = np.float32(0.0137)
    q_ref, amax_ref = oracle.quantize_with_scale(x, float(scale))
    q, amax = hg.quantize_e4m3_delayed(xt.cuda(), torch.tensor([scale], device="cuda"))
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert float(amax.item()) == amax_ref


def test_delayed_scaling_matches_two_pass_and_chains(cuda_device):
    """With the tensor's own amax/448 it reproduces the two-pass quantiser; amax_out feeds the
    next step's scale without a host round trip."""
    import hipgemm_b200 as hg
    xs = [torch.from_numpy(oracle.normal_f32(1 << 20, seed=s, stddev=1.0 + s)).cuda() for s in range(3)]
    q2, s2 = hg.quantize_e4m3(xs[0])
    q1, amax = hg.quantize_e4m3_delayed(xs[0], s2)
    assert torch.equal(q1, q2) and float(amax.item()) == float(xs[0].abs().max().item())
    scale = s2
    for x in xs[1:]:
        q, amax = hg.quantize_e4m3_delayed(x, scale)
        q_ref, a_ref = oracle.quantize_with_scale(x.cpu().numpy(), float(scale.item()))
        assert np.array_equal(q.cpu().numpy(), q_ref) and float(amax.item()) == a_ref
        scale = amax / 448.0
    assert hg.device_status() == 0
