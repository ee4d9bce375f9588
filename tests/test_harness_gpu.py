"""GPU runs of the C++ harness that mirrors the reference's test.cpp (tests/cpp/), and
the kernel against the committed golden fixtures (tests/golden/)."""
import glob
import os
import subprocess

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(HERE, "cpp", "test_gemm")
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


def _harness(*args):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-s", "-C", os.path.join(HERE, "cpp")], check=True)
    r = subprocess.run([BIN, *map(str, args)], capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout + r.stderr


def test_reference_harness_default_4096(cuda_device):
    """test.cpp's default case: 4096^3, both inputs seed 0, N(-1,1), unscaled, launched
    through the fp8_gemm_4wave_256x256x128<4096, 4096, 4096> drop-in."""
    rc, out = _harness()
    assert rc == 0 and "Test passed: 1" in out and "reference validator (test.cpp:32-47): pass" in out, out


@pytest.mark.parametrize("M,N,K", [(1000, 1032, 2064), (512, 512, 512)])
def test_reference_harness_scaled(cuda_device, M, N, K):
    rc, out = _harness(M, N, K, "scaled")
    assert rc == 0 and "Test passed: 1" in out, out


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_kernel_on_golden_fixture(cuda_device, path):
    import hipgemm_b200 as hg
    g = np.load(path)
    a = torch.from_numpy(g["A"]).cuda()
    b = torch.from_numpy(g["B"]).cuda()
    sa = torch.tensor([float(g["scale_a"])], dtype=torch.float32, device="cuda")
    sb = torch.tensor([float(g["scale_b"])], dtype=torch.float32, device="cuda")
    for config in range(len(hg.config_names())):
        c = hg.fp8_gemm_tn(a, b, sa, sb, config=config)
        got = c.view(torch.int16).cpu().numpy().view(np.uint16)
        assert oracle.validate(got, g["C"])[0] == 0, (path, config)


def test_cuda_graph_capture_and_replay(cuda_device):
    """After the first call on a device, the GEMM, the MX GEMM and the quantisers are plain
    stream operations: a CUDA graph captures them, and replays on new input bytes give the
    same bits as eager calls."""
    import hipgemm_b200 as hg
    M, N, K = 512, 768, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    xa = torch.randn(M, K, device="cuda", generator=g)
    xb = torch.randn(N, K, device="cuda", generator=g)
    # First calls on the device (one-time set-up happens outside the capture).
    qa, sa = hg.quantize_e4m3(xa)
    qb, sb = hg.quantize_e4m3(xb)
    c = hg.fp8_gemm_tn(qa, qb, sa, sb)
    ma, sfa = hg.quantize_mx_e4m3(xa)
    mb, sfb = hg.quantize_mx_e4m3(xb)
    cm = hg.fp8_gemm_tn_mx(ma, mb, sfa, sfb)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        hg.quantize_e4m3(xa, out=qa, scale=sa, stream=stream)
        hg.quantize_e4m3(xb, out=qb, scale=sb, stream=stream)
        hg.fp8_gemm_tn(qa, qb, sa, sb, out=c, stream=stream)
        hg.quantize_mx_e4m3(xa, out=ma, sf_out=sfa, stream=stream)
        hg.quantize_mx_e4m3(xb, out=mb, sf_out=sfb, stream=stream)
        hg.fp8_gemm_tn_mx(ma, mb, sfa, sfb, out=cm, stream=stream)
    for seed in (11, 12):
        g.manual_seed(seed)
        xa.copy_(torch.randn(M, K, device="cuda", generator=g))
        xb.copy_(torch.randn(N, K, device="cuda", generator=g))
        graph.replay()
        torch.cuda.synchronize()
        qa2, sa2 = hg.quantize_e4m3(xa)
        qb2, sb2 = hg.quantize_e4m3(xb)
        ma2, sfa2 = hg.quantize_mx_e4m3(xa)
        mb2, sfb2 = hg.quantize_mx_e4m3(xb)
        assert torch.equal(hg.fp8_gemm_tn(qa2, qb2, sa2, sb2).view(torch.int16), c.view(torch.int16))
        assert torch.equal(hg.fp8_gemm_tn_mx(ma2, mb2, sfa2, sfb2).view(torch.int16), cm.view(torch.int16))
    assert hg.device_status() == 0
