"""M-sharded multi-GPU FP8 GEMM: one process per GPU, torch.distributed for plumbing.

Rank r of P owns rows [r*M//P, (r+1)*M//P) of A and of C and a full copy of B, so the
GEMM itself needs no communication (each rank calls the single-GPU kernel on its
rows).  The one optional exchange is an all-gather of the bf16 C shards over NCCL
(NVLink / NVSwitch) into a full C on every rank.  The reference is single-GPU
(fp8_4wave.hpp:334-567 launched once at test.cpp:79); this module has no counterpart
there and follows the row partition the benchmark configs prescribe.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import check, lib
from .gemm import _check_operand, _ptr, _stream_handle, fp8_gemm_tn


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


class PeerCBuffers:
    """A full M x N bf16 C on every rank of `group`, each rank's buffer mapped into every
    other rank's process with CUDA IPC, for ShardedGemm.run_allgather.  Collective:
    every rank constructs it (and closes it) together."""

    def __init__(self, M: int, N: int, device: torch.device, group=None):
        self.M, self.N, self.group = M, N, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.local = torch.empty((M, N), dtype=torch.bfloat16, device=device)
        self._bases: list[int] = []
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_size_t(0)
        with torch.cuda.device(device):
            check(lib().hgemm_ipc_export(self.local.data_ptr(), handle, ctypes.byref(offset)), "hgemm_ipc_export")
        mine = (bytes(handle), int(offset.value))
        allh = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        ptrs = []
        for r, (h, off) in enumerate(allh):
            if r == self.rank:
                ptrs.append(self.local.data_ptr())
                continue
            base = ctypes.c_void_p(0)
            buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            with torch.cuda.device(device):
                check(lib().hgemm_ipc_import(buf, ctypes.byref(base)), "hgemm_ipc_import")
            self._bases.append(int(base.value))
            ptrs.append(int(base.value) + off)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)

    def close(self) -> None:
        """Unmaps the peers' buffers (call on every rank, after the last use)."""
        for b in self._bases:
            check(lib().hgemm_ipc_close(ctypes.c_void_p(b)), "hgemm_ipc_close")
        self._bases = []


def stream_barrier(group=None) -> None:
    """Orders a one-element NCCL all-reduce on the current stream: work queued after it
    starts only once every rank's preceding work has completed."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        t = torch.zeros(1, dtype=torch.float32, device=torch.cuda.current_device())
        dist.all_reduce(t, group=group)


def run_allgather(sg: ShardedGemm, a_rows: torch.Tensor, b: torch.Tensor, bufs: PeerCBuffers, scale_a=None,
                  scale_b=None, barrier: bool = True, barrier_before: bool = True) -> torch.Tensor:
    """This rank's rows of C = A . B^T computed and written into every rank's full C in
    one kernel (hgemm_fp8_tn_rows_allgather).

    The kernel writes into every peer's buffer, so two stream barriers bracket it:
    barrier_before=True orders it after every rank's work queued before this call (in
    particular any reads of the previous result: without it, this rank's stores could
    overwrite a peer's C while that peer is still reading it), and barrier=True orders every
    rank's stores before work queued after this call, so that bufs.local holds the whole C.
    Leave barrier_before on unless the caller orders its reads of the buffers against the
    next call some other way."""
    _check_operand("a_rows", a_rows)
    _check_operand("b", b)
    if tuple(a_rows.shape) != (sg.rows, sg.K) or tuple(b.shape) != (sg.N, sg.K):
        raise ValueError("shard shapes do not match the partition")
    if (bufs.M, bufs.N) != (sg.M, sg.N) or bufs.world != sg.world or bufs.rank != sg.rank:
        raise ValueError("buffers do not match the partition")
    # a_rows holds rows [row_begin, row_end): pass its pointer as the base of rows
    # [0, rows) of a virtual full A, i.e. shift by -row_begin rows.
    a_base = a_rows.data_ptr() - sg.row_begin * sg.K
    if barrier_before:
        stream_barrier(sg.group)
    with torch.cuda.device(a_rows.device):
        rc = lib().hgemm_fp8_tn_rows_allgather(a_base, _ptr(b), bufs.ptrs, sg.world, sg.rank, sg.M, sg.N, sg.K,
                                               sg.row_begin, sg.row_end, _ptr(scale_a), _ptr(scale_b),
                                               _stream_handle(None))
    check(rc, "hgemm_fp8_tn_rows_allgather")
    if barrier:
        stream_barrier(sg.group)
    return bufs.local
