"""Request sharding across ranks: pure logic plus world_size-2 gloo runs.

On CPU the per-rank compute is the oracle (test infrastructure standing in
for the GPU op); what is under test is the split, the rebasing of
``last_index`` and the local tile tables, and the gather back to rank 0.
"""

from __future__ import annotations

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import rope_oracle
from testfiles_b200 import sharding, workloads


def test_shard_tokens_covers_range_in_64_aligned_chunks():
    for n in (0, 1, 63, 64, 65, 16384, 16383, 9616):
        for world in (1, 2, 3, 4, 8):
            ranges = [sharding.shard_tokens(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0 and a0 <= a1
            for a0, a1 in ranges[:-1]:
                assert a0 % 64 == 0 and a1 % 64 == 0 or a1 == n


def test_shard_requests_partitions_and_balances():
    rng = random.Random(0)
    for _ in range(200):
        bs = rng.randint(1, 200)
        lens = [rng.randint(1, 500) for _ in range(bs)]
        for world in (1, 2, 4, 8):
            ranges = sharding.shard_requests(lens, world)
            assert ranges[0][0] == 0 and ranges[-1][1] == bs
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            total = sum(lens)
            for r0, r1 in ranges:  # each rank is within one request of its fair share
                load = sum(lens[r0:r1])
                assert load <= total / world + max(lens) + 1
    assert sharding.shard_requests([16384] * 4, 4) == [(0, 1), (1, 2), (2, 3), (3, 4)]


def test_local_batch_rebases_and_rebuilds_tiles():
    lens = workloads.reference_uneven_lens(16384, 128)
    last = rope_oracle.make_last_index(16384, 128, lens)
    for world in (1, 2, 4, 8):
        covered = []
        for r0, r1 in sharding.shard_requests(lens, world):
            local = sharding.local_batch(lens, (r0, r1), last)
            assert local.tile_starts == rope_oracle.build_tile_starts(lens[r0:r1])
            assert [v + local.token_begin for v in local.last_index] == last[r0:r1]
            covered.extend(range(local.token_begin, local.token_end))
        assert covered == list(range(16384))
    with pytest.raises(ValueError):
        sharding.local_batch([4, 4], (1, 2), [3, 3])  # index outside rank 1's tokens


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = workloads.find_case("b_mirror_segmented_n9616_bs16_uneven")
        full = workloads.make_inputs(case, "cpu")
        lens = case.segment_lens
        r0, r1 = sharding.shard_requests(lens, world)[rank]
        local = sharding.local_batch(lens, (r0, r1), full.last_index.tolist())
        t0, t1 = local.token_begin, local.token_end
        key = full.key[t0:t1].clone()
        query = full.query[r0:r1].clone()
        positions = full.positions[t0:t1]
        last = torch.tensor(local.last_index, dtype=torch.int64)
        # per-rank compute (the GPU op on a B200; the oracle here)
        q_out, k_out = rope_oracle.tiled_outputs(query, key, positions, full.cache, local.num_work_tiles, 1,
                                                 local.tile_starts, last)
        k_counts = [b.n_tokens for b in (sharding.local_batch(lens, rr) for rr in sharding.shard_requests(lens, world))]
        q_counts = [rr[1] - rr[0] for rr in sharding.shard_requests(lens, world)]
        k_all = sharding.gather_rows(k_out, k_counts)
        q_all = sharding.gather_rows(q_out, q_counts)
        if rank == 0:
            q_ref, k_ref = rope_oracle.reference_outputs(full.query, full.key, full.positions, full.last_index,
                                                         full.cache)
            queue.put((torch.equal(q_all, q_ref), torch.equal(k_all, k_ref)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_reassemble_unsharded_result():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    result = queue.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert result == (True, True)
