"""The allocation-free entry point hgemm_fp8_tn_static_scratch, called through the C ABI.

It is meant for callers that may not allocate device memory at all, for example an
engine that has already given all GPU memory to its own allocator, or a plugin host that
forbids driver allocations.  It keeps the stream-K scratch in a fixed 8 MiB array inside
the library, so two calls in a row reuse (and must correctly re-clear) the same memory,
and it must never create the library's workspace pool, not even on its first call.
This file is collected last on purpose: a failure here leaves every other test run.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _inputs(M, N, K, seed):
    A, sa = oracle.make_quantized((M, K), seed)
    B, sb = oracle.make_quantized((N, K), seed + 1)
    dev = torch.device("cuda:0")
    a = torch.from_numpy(A).to(dev)
    b = torch.from_numpy(B).to(dev)
    ta = torch.tensor([sa], dtype=torch.float32, device=dev)
    tb = torch.tensor([sb], dtype=torch.float32, device=dev)
    return A, B, sa, sb, a, b, ta, tb


def _bits(c: torch.Tensor) -> np.ndarray:
    return c.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("M,N,K", [(384, 640, 1536), (129, 264, 4112)])
def test_static_scratch_matches_oracle_and_existing_entry_point(cuda_device, M, N, K):
    """Two calls in a row through the allocation-free entry point, each checked against the
    CPU oracle and against hgemm_fp8_tn (the existing entry point) on the same inputs with
    the tests' tolerance |d| <= 1e-2*|ref| + 1e-3; the stream-K schedule must actually
    split tiles here, so the shared scratch really carries partial tiles."""
    import hipgemm_b200 as hg
    L = hg.lib()
    A, B, sa, sb, a, b, ta, tb = _inputs(M, N, K, seed=M + N)
    assert hg.plan(M, N, K, schedule=hg.HGEMM_SCHEDULE_STREAM_K)["sk_tiles"] > 0
    stream = torch.cuda.current_stream().cuda_stream
    ref_gpu = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    assert L.hgemm_fp8_tn(a.data_ptr(), b.data_ptr(), ref_gpu.data_ptr(), M, N, K, ta.data_ptr(), tb.data_ptr(),
                          stream) == hg.HGEMM_OK
    ref_cpu = oracle.gemm(A, B, sa, sb)
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = L.hgemm_fp8_tn_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, ta.data_ptr(),
                                           tb.data_ptr(), stream)
        assert rc == hg.HGEMM_OK, L.hgemm_error_string(rc)
        torch.cuda.synchronize()
        got = _bits(out)
        bad, first = oracle.validate(got, ref_cpu)
        assert bad == 0, f"{bad} elements outside tolerance of the oracle (first flat index {first})"
        bad, first = oracle.validate(got, _bits(ref_gpu))
        assert bad == 0, f"{bad} elements outside tolerance of hgemm_fp8_tn (first flat index {first})"
    assert hg.device_status() == 0


def test_static_scratch_refuses_problems_beyond_its_size(cuda_device):
    """A problem whose stream-K scratch exceeds the fixed array is refused up front."""
    import hipgemm_b200 as hg
    M, N, K = 1024, 8192, 8192
    assert hg.plan(M, N, K, schedule=hg.HGEMM_SCHEDULE_STREAM_K)["workspace_bytes"] > 8 << 20
    a = torch.zeros((M, K), dtype=torch.uint8, device="cuda")
    b = torch.zeros((N, K), dtype=torch.uint8, device="cuda")
    out = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    rc = hg.lib().hgemm_fp8_tn_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, None, None,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == hg.HGEMM_ERR_UNSUPPORTED


_FRESH_PROCESS = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    import torch
    import hipgemm_b200 as hg
    L = hg.lib()
    M, N, K = 384, 640, 1536
    a = torch.ones((M, K), dtype=torch.uint8, device="cuda")
    b = torch.ones((N, K), dtype=torch.uint8, device="cuda")
    c = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert L.hgemm_fp8_tn_static_scratch(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, None, None, s) == 0
    torch.cuda.synchronize()
    before = L.hgemm_debug_workspace_pool_created(0)
    # The same schedule without a workspace takes its scratch from the pool: created now.
    assert L.hgemm_fp8_tn_ex(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, None, None, s, 0,
                             hg.HGEMM_SCHEDULE_STREAM_K, None, 0) == 0
    torch.cuda.synchronize()
    after = L.hgemm_debug_workspace_pool_created(0)
    print("POOL", before, after)
""")


def test_static_scratch_first_calls_create_no_pool(cuda_device):
    """In a fresh process, the allocation-free entry point's first calls on a device leave the
    library's workspace pool uncreated; a stream-K call without a workspace then creates it."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    res = subprocess.run([sys.executable, "-c", _FRESH_PROCESS.format(root=ROOT)], capture_output=True, text=True,
                         timeout=300, env=env)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "POOL 0 1" in res.stdout, res.stdout + res.stderr
