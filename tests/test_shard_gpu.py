"""M-sharded multi-GPU GEMM on real GPUs: one process per GPU over NCCL.  Each rank runs
the sm_100a kernel on its rows (B replicated) and the bf16 C shards are all-gathered; the
result must equal the single-GPU product bit for bit (row shards do not change any
element's accumulation).  Skipped when fewer than two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import oracle
        from hipgemm_b200 import fp8_gemm_tn
        from hipgemm_b200.shard import ShardedGemm
        A, sa = oracle.make_quantized((M, K), 0)
        B, sb = oracle.make_quantized((N, K), 1)
        sg = ShardedGemm(M, N, K)
        a = torch.from_numpy(np.ascontiguousarray(A[sg.row_begin:sg.row_end])).to(dev)
        b = torch.from_numpy(B).to(dev)
        ta = torch.tensor([sa], dtype=torch.float32, device=dev)
        tb = torch.tensor([sb], dtype=torch.float32, device=dev)
        c_rows = sg.run(a, b, ta, tb)
        full = sg.all_gather(c_rows)
        torch.cuda.synchronize()
        if rank == 0:
            single = fp8_gemm_tn(torch.from_numpy(A).to(dev), b, ta, tb)
            same = torch.equal(full.view(torch.int16), single.view(torch.int16))
            got = full.view(torch.int16).cpu().numpy().view(np.uint16)
            rows = np.array([0, M // 3, M - 1], dtype=np.int32)
            ok_oracle = oracle.validate(got[rows], oracle.gemm_rows(A, B, rows, sa, sb))[0] == 0
            np.save(os.path.join(out_dir, "ok.npy"), np.array([same, ok_oracle]))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(4096, 2048, 1024), (1000, 1032, 528)])
def test_sharded_gemm_matches_single_gpu(tmp_path, M, N, K):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    same, ok_oracle = np.load(tmp_path / "ok.npy")
    assert same and ok_oracle


def _fused_worker(rank, world, port, M, N, K, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    bufs = None
    try:
        import oracle
        import hipgemm_b200 as hg
        from hipgemm_b200.shard import PeerCBuffers, ShardedGemm, run_allgather, stream_barrier
        A, sa = oracle.make_quantized((M, K), 0)
        B, sb = oracle.make_quantized((N, K), 1)
        sg = ShardedGemm(M, N, K)
        a = torch.from_numpy(np.ascontiguousarray(A[sg.row_begin:sg.row_end])).to(dev)
        b = torch.from_numpy(B).to(dev)
        ta = torch.tensor([sa], dtype=torch.float32, device=dev)
        tb = torch.tensor([sb], dtype=torch.float32, device=dev)
        bufs = PeerCBuffers(M, N, dev)
        single = hg.fp8_gemm_tn(torch.from_numpy(A).to(dev), b, ta, tb)
        ok = True
        for step in range(2):  # twice: the buffers are rewritten in place
            bufs.local.fill_(float("nan"))
            # run_allgather's barrier_before: nobody writes into a buffer before its owner
            # has cleared it (and, in a real loop, finished reading the previous result).
            full = run_allgather(sg, a, b, bufs, ta, tb)
            torch.cuda.synchronize()
            ok = ok and torch.equal(full.view(torch.int16), single.view(torch.int16))
        ok = ok and hg.device_status() == 0
        np.save(os.path.join(out_dir, f"fused{rank}.npy"), np.array([ok]))
        stream_barrier()
        torch.cuda.synchronize()
    finally:
        if bufs is not None:
            bufs.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(4096, 2048, 1024), (1000, 1032, 528)])
def test_fused_allgather_gives_every_rank_the_full_product(tmp_path, M, N, K):
    """GEMM + all-gather in one kernel: every rank's C buffer equals the single-GPU C."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    mp.start_processes(_fused_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert bool(np.load(tmp_path / f"fused{r}.npy")[0]), f"rank {r}"
