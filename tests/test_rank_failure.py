"""Failure detection across ranks, made on the host (gloo ranks on CPU).

Three failures, none of which touches a GPU:

* a rank's C-ABI call fails (the real library's host validation refuses a
  negative token count, which needs no device): :func:`sharding.check_all_ranks`
  raises the same :class:`sharding.RankFailure` on every rank and no rank
  enters the gather;
* a rank dies before the status step: the survivor's collective ends with an
  error within the process group's short timeout instead of waiting for good;
* a rank never joins: the survivor's rendezvous times out.
"""

from __future__ import annotations

import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PG_TIMEOUT = datetime.timedelta(seconds=5)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=PG_TIMEOUT)


def _reported_failure(rank: int, world: int, port: int, queue) -> None:
    from testfiles_b200 import _native, sharding

    _init(rank, world, port)
    try:
        if rank == 1:
            # the library refuses the call on the host, before any CUDA work
            rc = _native.load().welm_rope_ordinary(None, None, None, None, None, 0, -1, 1536, 256, 0, 16, None, None)
        else:
            rc = 0
        gathered = False
        try:
            sharding.check_all_ranks(rc << 8)
            sharding.gather_rows(torch.zeros(1, 4), [1] * world)
            gathered = True
        except sharding.RankFailure as err:
            queue.put((rank, "failure", err.status, gathered))
        else:
            queue.put((rank, "ok", 0, gathered))
        dist.barrier()  # both ranks are still in step after the failure
    finally:
        dist.destroy_process_group()


def _dead_rank(rank: int, world: int, port: int, queue) -> None:
    from testfiles_b200 import sharding

    phase, t0 = "init", time.monotonic()
    try:
        _init(rank, world, port)
        phase = "first step"
        dist.barrier()  # both ranks are fully connected and one step is done
        if rank == 1:
            time.sleep(0.5)  # let the survivor enter its next collective
            os._exit(7)  # dies between steps: nothing of it is in flight
        phase, t0 = "status step", time.monotonic()
        sharding.check_all_ranks(0)
        queue.put((rank, phase, "no error", time.monotonic() - t0))
    except Exception as err:  # gloo reports a closed peer or a timeout
        queue.put((rank, phase, type(err).__name__, time.monotonic() - t0))
    queue.close()
    queue.join_thread()  # the report must reach the pipe before the hard exit below
    os._exit(0)  # the group cannot be torn down cleanly with a peer gone


def _never_joins(rank: int, world: int, port: int, queue) -> None:
    if rank == 1:
        return
    t0 = time.monotonic()
    try:
        _init(rank, world, port)
        queue.put((rank, "joined", time.monotonic() - t0))
    except Exception as err:
        queue.put((rank, type(err).__name__, time.monotonic() - t0))


def _run(target, world: int = 2, expect: int = 1, join_s: float = 60.0):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [queue.get(timeout=120) for _ in range(expect)]
    finally:
        for p in procs:
            p.join(timeout=join_s)
            if p.is_alive():  # the exact child this test started
                p.kill()
                p.join(timeout=10)
    return sorted(results), [p.exitcode for p in procs]


def test_reported_failure_reaches_every_rank_and_skips_the_gather():
    from testfiles_b200 import _native

    results, codes = _run(_reported_failure, expect=2)
    status = _native.ERR_BAD_SIZE << 8
    assert results == [(0, "failure", status, False), (1, "failure", status, False)]
    assert codes == [0, 0]


def test_dead_rank_ends_the_survivors_collective_with_an_error():
    results, codes = _run(_dead_rank)
    (rank, phase, outcome, elapsed), = results
    assert (rank, phase) == (0, "status step") and outcome != "no error"
    assert elapsed < 60, f"the survivor waited {elapsed:.0f} s"
    assert codes == [0, 7]


def test_rank_that_never_joins_times_out_the_rendezvous():
    results, codes = _run(_never_joins)
    (rank, outcome, elapsed), = results
    assert rank == 0 and outcome != "joined"
    assert elapsed < 60
    assert codes == [0, 0]
