"""Host logic of the M-sharded multi-GPU path, on CPU with gloo (world size 2 and 3):
the row partition, the global per-tensor scale, and the all-gather that assembles C.
The per-rank GEMM is stood in for by the CPU oracle (test infrastructure) since there
is no GPU here; on a GPU box the same ShardedGemm calls the sm_100a kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hipgemm_b200.shard import ShardedGemm, max_rows, row_range


@pytest.mark.parametrize("M,P", [(8192, 1), (8192, 8), (16384, 8), (4000, 3), (7, 4), (1, 2), (0, 2), (129, 8)])
def test_row_range_partitions_m(M, P):
    ranges = [row_range(M, r, P) for r in range(P)]
    assert ranges[0][0] == 0 and ranges[-1][1] == M
    for (a0, a1), (b0, b1) in zip(ranges[:-1], ranges[1:]):
        assert a1 == b0
    sizes = [r1 - r0 for r0, r1 in ranges]
    assert max(sizes) - min(sizes) <= 1 and max_rows(M, P) == max(sizes)


def test_row_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        from hipgemm_b200.shard import global_amax_scale
        # Full inputs are generated identically on every rank; each keeps its rows of A.
        x_full = torch.from_numpy(oracle.normal_f32(M * K, 5)).view(M, K)
        sg = ShardedGemm(M, N, K)
        x_rows = x_full[sg.row_begin:sg.row_end]
        scale = global_amax_scale(x_rows)
        expect = np.float32(np.abs(x_full.numpy()).max()) / np.float32(448.0)
        assert float(scale) == pytest.approx(float(expect), rel=0, abs=0)
        A_full = oracle.quantize(x_full.numpy())[0]
        B, sb = oracle.make_quantized((N, K), 6)
        sa = float(scale)
        C_rows = oracle.gemm(np.ascontiguousarray(A_full[sg.row_begin:sg.row_end]), B, sa, sb) if sg.rows else \
            np.empty((0, N), np.uint16)
        c = torch.from_numpy(C_rows.view(np.int16)).view(torch.bfloat16)
        full = sg.all_gather(c)
        assert tuple(full.shape) == (M, N)
        ref = oracle.gemm(A_full, B, sa, sb)
        got = full.view(torch.int16).numpy().view(np.uint16)
        np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array([np.array_equal(got, ref)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M", [(2, 64), (2, 37), (3, 50)])
def test_sharded_gather_reassembles_full_product(tmp_path, world, M):
    N, K = 24, 64
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert bool(np.load(tmp_path / f"ok{r}.npy")[0]), f"rank {r}"
