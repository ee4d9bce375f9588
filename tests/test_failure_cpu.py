"""Failure detection of the multi-rank host path, with the failure made on the host (gloo ranks
on CPU; no GPU is faulted, trapped or hung).

- A rank that never joins: the others' rendezvous ends with an error after the process-group
  timeout instead of waiting for ever.
- A rank that fails between steps, before the all-gather of C: the surviving rank's
  ShardedGemm.all_gather raises (peer gone or timeout) instead of hanging, and the error
  reaches the caller.

Each rank runs in its own spawned process with a hard limit on how long the test waits for it.
"""
import datetime
import multiprocessing as mp
import os
import socket
import time

import pytest

PG_TIMEOUT_S = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _write(out_dir: str, rank: int, text: str) -> None:
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(text)


def _lonely_rank(port: int, out_dir: str) -> None:
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    except Exception as e:  # the expected outcome: rank 1 never arrives
        _write(out_dir, 0, f"raised {type(e).__name__} after {time.monotonic() - t0:.1f}s")
        return
    _write(out_dir, 0, "joined")
    dist.destroy_process_group()


def test_rank_that_never_joins_ends_the_rendezvous_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), str(tmp_path)))
    p.start()
    p.join(120)
    if p.is_alive():
        p.kill()
        p.join()
        pytest.fail("the rendezvous did not end within 120 s")
    text = (tmp_path / "rank0.txt").read_text()
    assert text.startswith("raised"), text


def _rank_with_failure(rank: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    from hipgemm_b200.shard import ShardedGemm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    M, N, K = 64, 16, 32
    sg = ShardedGemm(M, N, K)
    if rank == 1:
        # The injected failure: this rank leaves between steps, before the all-gather, with
        # none of its work in flight.
        _write(out_dir, 1, "left")
        os._exit(3)
    c_rows = torch.zeros((sg.rows, N), dtype=torch.bfloat16)
    t0 = time.monotonic()
    try:
        sg.all_gather(c_rows)
    except Exception as e:  # the expected outcome: the peer is gone
        _write(out_dir, 0, f"raised {type(e).__name__} after {time.monotonic() - t0:.1f}s")
        os._exit(0)
    _write(out_dir, 0, "gathered")
    os._exit(0)


def test_rank_failing_before_the_all_gather_surfaces_as_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_with_failure, args=(r, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 120
    for p in procs:
        p.join(max(1.0, deadline - time.monotonic()))
    hung = [i for i, p in enumerate(procs) if p.is_alive()]
    for i in hung:
        procs[i].kill()
        procs[i].join()
    assert not hung, f"ranks {hung} did not end within 120 s"
    assert (tmp_path / "rank1.txt").read_text() == "left"
    text = (tmp_path / "rank0.txt").read_text()
    assert text.startswith("raised"), text
