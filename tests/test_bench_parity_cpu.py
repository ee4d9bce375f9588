"""bench.py's post-run parity check at N > 1, on CPU with gloo (world size 2 and 3): the
gather of A's row shards, the single-call comparison of every rank's block, the all-gather of
C and rank 0's oracle rows.  The per-rank GEMM is stood in for by the CPU oracle (test
infrastructure; there is no GPU here), so a clean run must report zero mismatches, and a
planted error in one rank's block (planted in the oracle stand-in's output, on the CPU) must
be counted."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
import oracle
from hipgemm_b200.shard import ShardedGemm


class _OracleGemm:
    """Stands in for hipgemm_b200 in bench.parity_check: fp8_gemm_tn on CPU tensors."""

    @staticmethod
    def fp8_gemm_tn(a, b, sa, sb):
        bits = oracle.gemm(a.numpy(), b.numpy(), float(sa.item()), float(sb.item()))
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, plant, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sg = ShardedGemm(M, N, K)
        A, sa = oracle.make_quantized((M, K), 3)
        B, sb = oracle.make_quantized((N, K), 4)
        a_rows = torch.from_numpy(np.ascontiguousarray(A[sg.row_begin:sg.row_end]))
        b = torch.from_numpy(B)
        ta = torch.tensor([sa], dtype=torch.float32)
        tb = torch.tensor([sb], dtype=torch.float32)
        c_rows = _OracleGemm.fp8_gemm_tn(a_rows, b, ta, tb).clone()
        if plant and rank == world - 1:
            # Corrupt the block's last row (always one of the oracle-checked rows).
            c_rows[-1, 5] = torch.tensor(1234.0, dtype=torch.bfloat16)
        out = bench.parity_check(_OracleGemm, sg, a_rows, b, ta, tb, c_rows, torch.device("cpu"), world, rank)
        if rank == 0:
            np.save(os.path.join(out_dir, "parity.npy"),
                    np.array([out["rows_checked"], out["mismatches"], out["bitwise_vs_single_gpu"]["block_mismatched"],
                              out["bitwise_vs_single_gpu"]["nccl_allgather_mismatched"]]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K,world", [(512, 256, 256, 2), (390, 136, 128, 3)])
@pytest.mark.parametrize("plant", [False, True])
def test_parity_check_counts_mismatches_across_ranks(tmp_path, M, N, K, world, plant):
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, plant, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    rows, bad_oracle, bad_block, bad_gather = np.load(tmp_path / "parity.npy")
    assert rows == len(bench.parity_rows(M, world))
    if plant:
        assert bad_oracle == 1 and bad_block == 1 and bad_gather == world  # every rank gathers the bad row
    else:
        assert bad_oracle == 0 and bad_block == 0 and bad_gather == 0
