"""M-sharded multi-GPU FP8 GEMM: one process per GPU, torch.distributed for plumbing.

Rank r of P owns rows [r*M//P, (r+1)*M//P) of A and of C and a full copy of B, so the
GEMM itself needs no communication (each rank calls the single-GPU kernel on its
rows).  The one optional exchange is an all-gather of the bf16 C shards over NCCL
(NVLink / NVSwitch) into a full C on every rank.  The reference is single-GPU
(fp8_4wave.hpp:334-567 launched once at test.cpp:79); this module has no counterpart
there and follows the row partition the benchmark configs prescribe.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .gemm import fp8_gemm_tn


def row_range(M: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced row block of `rank` (sizes differ by at most one row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return rank * M // world, (rank + 1) * M // world


def max_rows(M: int, world: int) -> int:
    return max(r1 - r0 for r0, r1 in (row_range(M, r, world) for r in range(world)))


def global_amax_scale(x_local: torch.Tensor, group=None) -> torch.Tensor:
    """Per-tensor scale amax/448 of a row-sharded tensor: local amax, all-reduce MAX.
    Every rank gets the same fp32 scale (shape [1])."""
    amax = x_local.detach().abs().amax().float().reshape(1)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))


class ShardedGemm:
    """C = A . B^T with A and C split by rows across the ranks of `group`.

    run() computes this rank's rows; all_gather() assembles the full C on every rank.
    Uneven splits are padded to the largest shard for the collective, then trimmed.
    """

    def __init__(self, M: int, N: int, K: int, group=None):
        self.M, self.N, self.K = M, N, K
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.row_begin, self.row_end = row_range(M, self.rank, self.world)
        self.rows = self.row_end - self.row_begin
        self.pad_rows = max_rows(M, self.world)

    def run(self, a_rows: torch.Tensor, b: torch.Tensor, scale_a=None, scale_b=None, out=None, config: int = 0):
        if tuple(a_rows.shape) != (self.rows, self.K) or tuple(b.shape) != (self.N, self.K):
            raise ValueError("shard shapes do not match the partition")
        return fp8_gemm_tn(a_rows, b, scale_a, scale_b, out=out, config=config)

    def gather_buffer(self, device) -> torch.Tensor:
        return torch.empty((self.world * self.pad_rows, self.N), dtype=torch.bfloat16, device=device)

    def all_gather(self, c_rows: torch.Tensor, gathered: torch.Tensor | None = None) -> torch.Tensor:
        """Full M x N C on every rank from each rank's (rows x N) shard."""
        if gathered is None:
            gathered = self.gather_buffer(c_rows.device)
        if self.rows == self.pad_rows:
            src = c_rows
        else:
            src = torch.zeros((self.pad_rows, self.N), dtype=c_rows.dtype, device=c_rows.device)
            src[: self.rows].copy_(c_rows)
        if self.world == 1:
            gathered[: self.rows].copy_(src[: self.rows])
        else:
            dist.all_gather_into_tensor(gathered, src.contiguous(), group=self.group)
        if all(row_range(self.M, r, self.world)[1] - row_range(self.M, r, self.world)[0] == self.pad_rows
               for r in range(self.world)):
            return gathered[: self.M]
        parts = []
        for r in range(self.world):
            r0, r1 = row_range(self.M, r, self.world)
            parts.append(gathered[r * self.pad_rows: r * self.pad_rows + (r1 - r0)])
        return torch.cat(parts, dim=0)
