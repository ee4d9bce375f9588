"""The allocation-free entry point hgemm_fp8_tn_static_scratch, called through the C ABI.

It is meant for callers that may not allocate device memory at all, for example an
engine that has already given all GPU memory to its own allocator, or a plugin host that
forbids driver allocations.  It keeps the stream-K scratch in a fixed 8 MiB array inside
the library, so two calls in a row reuse (and must correctly re-clear) the same memory.
This file is collected last on purpose: a failure here leaves every other test run.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _entry():
    import hipgemm_b200 as hg
    fn = hg.lib().hgemm_fp8_tn_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 3
    return fn


def _inputs(M, N, K, seed):
    A, sa = oracle.make_quantized((M, K), seed)
    B, sb = oracle.make_quantized((N, K), seed + 1)
    dev = torch.device("cuda:0")
    a = torch.from_numpy(A).to(dev)
    b = torch.from_numpy(B).to(dev)
    ta = torch.tensor([sa], dtype=torch.float32, device=dev)
    tb = torch.tensor([sb], dtype=torch.float32, device=dev)
    return a, b, ta, tb


def _bits(c: torch.Tensor) -> np.ndarray:
    return c.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("M,N,K", [(384, 640, 1536), (129, 264, 4112)])
def test_static_scratch_matches_existing_entry_point(cuda_device, M, N, K):
    """Two calls in a row through the allocation-free entry point, each checked against
    hgemm_fp8_tn (the existing entry point) on the same inputs with the tests' tolerance
    |d| <= 1e-2*|ref| + 1e-3; the stream-K schedule must actually split tiles here."""
    import hipgemm_b200 as hg
    fn = _entry()
    a, b, ta, tb = _inputs(M, N, K, seed=M + N)
    assert hg.plan(M, N, K, schedule=hg.HGEMM_SCHEDULE_STREAM_K)["sk_tiles"] > 0
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    assert hg.lib().hgemm_fp8_tn(a.data_ptr(), b.data_ptr(), ref.data_ptr(), M, N, K, ta.data_ptr(),
                                 tb.data_ptr(), stream) == hg.HGEMM_OK
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = fn(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, ta.data_ptr(), tb.data_ptr(), stream)
        assert rc == hg.HGEMM_OK, hg.lib().hgemm_error_string(rc)
        torch.cuda.synchronize()
        bad, first = oracle.validate(_bits(out), _bits(ref))
        assert bad == 0, f"{bad} elements outside tolerance (first flat index {first})"
    assert hg.device_status() == 0


def test_static_scratch_refuses_problems_beyond_its_size(cuda_device):
    """A problem whose stream-K scratch exceeds the fixed array is refused up front."""
    import hipgemm_b200 as hg
    fn = _entry()
    M, N, K = 1024, 8192, 8192
    assert hg.plan(M, N, K, schedule=hg.HGEMM_SCHEDULE_STREAM_K)["workspace_bytes"] > 8 << 20
    a = torch.zeros((M, K), dtype=torch.uint8, device="cuda")
    b = torch.zeros((N, K), dtype=torch.uint8, device="cuda")
    out = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    rc = fn(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, None, None, torch.cuda.current_stream().cuda_stream)
    assert rc == hg.HGEMM_ERR_UNSUPPORTED
