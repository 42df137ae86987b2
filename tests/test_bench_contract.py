"""CPU checks of the figures bench.py reports beside its timing: the
algorithmic byte count, the ncu traffic figure it reads from the committed
profile, the published figure behind vs_baseline, and the result-line
configuration."""

from __future__ import annotations

import importlib.util

from conftest import REPO
from testfiles_b200 import workloads


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_algorithmic_bytes_match_the_workload_model():
    bench = load_bench()
    case = workloads.find_case("b_prefill_m16384")
    assert bench.algorithmic_bytes(bench.TOKENS) == workloads.min_bytes(case) == 33_685_504


def test_traffic_figure_comes_from_the_committed_profile():
    bench = load_bench()
    traffic, source = bench.profiled_traffic()
    assert traffic is not None
    # DRAM bytes per launch close to the algorithmic reads (writes stay in L2)
    assert 19_000_000 <= traffic <= 19_100_000
    # the line says where the figure comes from: a separate capture, not this run
    assert "profiles/rope_ordinary_prefill_m16384.md" in source and "not measured by this run" in source


def test_vs_baseline_uses_the_published_figure():
    bench = load_bench()
    assert abs(bench.PUBLISHED_GBS - bench.algorithmic_bytes(bench.TOKENS) / 38.69e-6 / 1e9) < 1.0
    assert "38.69" in bench.PUBLISHED_SOURCE


def test_result_line_configuration():
    bench = load_bench()
    cfg = bench.workload_config(4)
    assert cfg["global_tokens"] == 4 * bench.TOKENS and cfg["parallelism"] == "request-sharded dp4"
    assert bench.BUFFER_SETS * bench.algorithmic_bytes(bench.TOKENS) > 2 * 126 * 1024 * 1024
    assert set(bench.OTHER_CONFIGS) <= {c.name for c in workloads.baseline_cases()}


def test_sharded_outputs_concatenate_to_the_golden_digests():
    """The bench checks multi-GPU legs by gathering each rank's rows and
    comparing their SHA-256 with the unsharded golden digest.  That only works
    if the shards' outputs, concatenated in rank order, are the unsharded
    outputs: checked here with the oracle on the CPU for the request-sharded
    segmented mirror and the token-sharded prefill at 1, 2, 3 and 8 ranks."""
    import torch

    from oracle import rope_oracle
    from testfiles_b200 import sharding

    bench = load_bench()
    case = workloads.find_case(bench.MIRROR_CASE)
    full = workloads.make_inputs(case, "cpu")
    want = bench.golden_outputs(bench.MIRROR_CASE)
    for world in (1, 2, 3, 8):
        qs, ks = [], []
        for rr in sharding.shard_requests(case.segment_lens, world):
            b = sharding.local_batch(case.segment_lens, rr, full.last_index.tolist())
            t0, t1 = b.token_begin, b.token_end
            q, k = rope_oracle.tiled_outputs(full.query[rr[0]:rr[1]], full.key[t0:t1], full.positions[t0:t1],
                                             full.cache, b.num_work_tiles, 1, b.tile_starts,
                                             torch.tensor(b.last_index))
            qs.append(q)
            ks.append(k)
        assert bench.sha256_rows(torch.cat(qs)) == want["query"], world
        assert bench.sha256_rows(torch.cat(ks)) == want["key"], world
    case = workloads.find_case(bench.PREFILL_CASE)
    full = workloads.make_inputs(case, "cpu")
    want = bench.golden_outputs(bench.PREFILL_CASE)
    for world in (2, 8):
        qs, ks = [], []
        for r in range(world):
            t0, t1 = sharding.shard_tokens(bench.TOKENS, world, r)
            q, k = rope_oracle.reference_outputs(full.query[t0:t1], full.key[t0:t1], full.positions[t0:t1], None,
                                                 full.cache)
            qs.append(q)
            ks.append(k)
        assert bench.sha256_rows(torch.cat(qs)) == want["query"], world
        assert bench.sha256_rows(torch.cat(ks)) == want["key"], world


def _rank_helpers_worker(rank: int, world: int, port: int, queue) -> None:
    import os

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench = load_bench()
        own = 5.0 + rank  # each rank's own timing
        top = bench.max_over_ranks(dist, own, torch.device("cpu"))
        every = bench.all_ranks(dist, own, torch.device("cpu"))
        queue.put((rank, top, every))
    finally:
        dist.destroy_process_group()


def test_rank_timing_helpers_over_two_gloo_ranks():
    """The max over ranks and every rank's own value, as the bench's timed
    legs report them, are the same on both ranks of a world_size-2 group."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank_helpers_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == [(0, 6.0, [5.0, 6.0]), (1, 6.0, [5.0, 6.0])]
    assert load_bench().all_ranks(None, 3.5, None) == [3.5]
