"""Request-sharded data parallelism on 2 GPUs (NCCL): each rank rotates its
shard with the sm_100a op, results are gathered to rank 0 and must equal the
oracle on the unsharded batch bit for bit.  Needs two visible GPUs."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    results = {}
    try:
        import testfiles_b200 as welm
        from oracle import rope_oracle
        from testfiles_b200 import sharding, workloads

        # segmented KV mirror, sharded by whole requests
        case = workloads.find_case("b_mirror_segmented_n16384_bs128_uneven")
        full = workloads.make_inputs(case, "cpu")
        lens = case.segment_lens
        ranges = sharding.shard_requests(lens, world)
        local = sharding.local_batch(lens, ranges[rank], full.last_index.tolist())
        r0, r1 = ranges[rank]
        t0, t1 = local.token_begin, local.token_end
        q = full.query[r0:r1].to(dev)
        k = full.key[t0:t1].to(dev)
        pos = full.positions[t0:t1].to(dev)
        last = torch.tensor(local.last_index, dtype=torch.int64, device=dev)
        starts = torch.tensor(local.tile_starts, dtype=torch.int32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        welm.welmv4_inplace_rope_npu(q, k, pos, full.cache.to(dev), last, starts, status=status)
        # every rank learns of any rank's device status before the gather
        sharding.check_all_ranks(int(status.item()), device=dev)
        k_counts = [sharding.local_batch(lens, rr).n_tokens for rr in ranges]
        q_counts = [rr[1] - rr[0] for rr in ranges]
        k_all = sharding.gather_rows(k, k_counts)
        q_all = sharding.gather_rows(q, q_counts)
        if rank == 0:
            q_ref, k_ref = rope_oracle.reference_outputs(full.query, full.key, full.positions, full.last_index,
                                                         full.cache)
            results["mirror"] = (torch.equal(q_all.cpu().view(torch.int16), q_ref.view(torch.int16)),
                                 torch.equal(k_all.cpu().view(torch.int16), k_ref.view(torch.int16)))

        # ordinary prefill, sharded by 64-aligned token ranges
        case = workloads.find_case("b_prefill_m9616")
        full = workloads.make_inputs(case, "cpu")
        a, b = sharding.shard_tokens(case.n_tokens, world, rank)
        q = full.query[a:b].to(dev)
        k = full.key[a:b].to(dev)
        welm.welmv4_inplace_rope_npu(q, k, full.positions[a:b].to(dev), full.cache.to(dev))
        counts = [sharding.shard_tokens(case.n_tokens, world, r)[1] - sharding.shard_tokens(case.n_tokens, world, r)[0]
                  for r in range(world)]
        q_all = sharding.gather_rows(q, counts)
        k_all = sharding.gather_rows(k, counts)
        if rank == 0:
            q_ref, k_ref = rope_oracle.reference_outputs(full.query, full.key, full.positions, None, full.cache)
            results["prefill"] = (torch.equal(q_all.cpu().view(torch.int16), q_ref.view(torch.int16)),
                                  torch.equal(k_all.cpu().view(torch.int16), k_ref.view(torch.int16)))
            queue.put(results)
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_request_sharding_matches_oracle():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = queue.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {"mirror": (True, True), "prefill": (True, True)}


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ops_on_a_device_that_is_not_current():
    """Tensors on cuda:1 while cuda:0 is current: every op runs on the tensors'
    device, equals the oracle, and leaves the caller's current device alone."""
    import testfiles_b200 as welm
    from oracle import rope_oracle
    from testfiles_b200 import workloads

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 1)

    case = workloads.find_case("b_prefill_m577")
    inp = workloads.make_inputs(case, "cpu")
    d = inp.to(dev)
    welm.welmv4_inplace_rope_npu(d.query, d.key, d.positions, d.cache)
    torch.cuda.synchronize(dev)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert torch.equal(d.query.cpu().view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(d.key.cpu().view(torch.int16), k_ref.view(torch.int16))

    case = workloads.find_case("b_mirror_segmented_n8192_bs8_uneven")
    inp = workloads.make_inputs(case, "cpu")
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    d = inp.to(dev)
    welm.welmv4_inplace_rope_npu(d.query, d.key, d.positions, d.cache, d.last_index, d.segment_tile_starts)
    torch.cuda.synchronize(dev)
    assert torch.equal(d.query.cpu().view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(d.key.cpu().view(torch.int16), k_ref.view(torch.int16))

    lens = torch.tensor(case.segment_lens, dtype=torch.int64, device=dev)
    d = inp.to(dev)
    welm.rope_mirror_from_lens(d.query, d.key, d.positions, d.cache, lens)
    torch.cuda.synchronize(dev)
    assert torch.equal(d.query.cpu().view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(d.key.cpu().view(torch.int16), k_ref.view(torch.int16))

    starts, num_tiles, last = welm.build_segment_tile_starts_device(lens, 8192 // 64 + len(case.segment_lens) + 1)
    host_starts, host_tiles, host_last = welm.build_segment_tile_starts(case.segment_lens)
    assert starts.device == dev and int(num_tiles.item()) == host_tiles
    assert torch.equal(starts[: host_tiles + 1].cpu(), host_starts)
    assert torch.equal(last.cpu(), host_last)

    from testfiles_b200 import host

    case = workloads.find_case("b_prefill_m577")
    inp = workloads.make_inputs(case, "cpu")
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    for transport in ("mapped", "staged"):
        q, k, p = inp.query.clone().pin_memory(), inp.key.clone().pin_memory(), inp.positions.pin_memory()
        host.welmv4_inplace_rope_host(q, k, p, inp.cache.to(dev), chunk_tokens=256, transport=transport)
        torch.cuda.synchronize(dev)
        assert torch.equal(q.view(torch.int16), q_ref.view(torch.int16)), transport
        assert torch.equal(k.view(torch.int16), k_ref.view(torch.int16)), transport
    assert torch.cuda.current_device() == 0
