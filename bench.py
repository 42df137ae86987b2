#!/usr/bin/env python3
"""Benchmark: WeLMv4 in-place partial RoPE, ordinary prefill M=16384, BF16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one launch of the op over one batch: Q bf16 [16384, 6, 256] and
K bf16 [16384, 1, 256] rotated in place at positions 0..16383 with an FP32
cos/sin cache [16384, 64] (rotary base 1e4), seeded N(0,1) synthetic data.

* ``value``: whole-job throughput in GB/s of ALGORITHMIC bytes (2056 B per
  token: Q 6 and K 1 rope slices read + written, one 256-B cos/sin row and an
  8-B position per token), with inputs resident in HBM.  K launches are
  replayed from a CUDA graph over 8 rotating buffer sets (270 MB touched
  between reuses, > 126 MB L2) and timed with CUDA events on the launching
  stream; multi-GPU runs take the max time over ranks.
* ``e2e``: the same metric through the public host-memory API
  ``welmv4_inplace_rope_host`` with pinned HOST buffers: every step reads
  the rotated lanes of Q and K and the positions from host memory over PCIe,
  rotates them and writes the lanes back to host memory (the mapped
  transport: one kernel whose reads and writes use both bus directions at
  once), all inside the timed region.  The staged copy pipeline and the
  whole-tensor-copy variant are reported beside it.
* ``roofline``: the op kernel's achieved GB/s (algorithmic bytes per launch
  over the average launch time of the graph-replayed region) against the
  measured HBM copy peak.
* ``cpu_baseline`` (rank 0, N=1 only): the reference's CPU algorithm (the
  oracle port of its torch path) on this host's cores, same workload.
* ``other_configs`` (rank 0, N=1 only): one configuration of each other
  benchmark family (prefill M=8192, decode M=1 and M=128, contiguous and
  segmented KV mirror at N=16384) and the KV mirror fused with the paged
  KV-cache write (N=16384, BS=128), timed after the headline, with a
  same-size device copy beside each (``--no-config-sweep`` skips it).

``--impl reference`` times the reference's CPU implementation alone (rank 0;
other ranks exit 0).  Multi-GPU runs (torchrun) shard requests: each rank
rotates its own 16384-token request (weak scaling); there is no collective
in the timed region.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from testfiles_b200.clocks import ClockSampler  # noqa: E402

METRIC = "µs/launch and achieved HBM GB/s (% of roofline) for M=16384 BF16 prefill RoPE"
TOKENS = 16384
BUFFER_SETS = 8
GRAPH_LAUNCHES = 64
FALLBACK_HBM_GBS = 6650.0
PROFILE_SUMMARY = REPO / "profiles" / "rope_ordinary_prefill_m16384.md"
REFERENCE_BUDGET_S = 60.0

# The reference's own published figure for this metric: prefill M=16384 with
# its tiled candidate kernel took 38.69 us per launch (NPU event timing on an
# Ascend 950PR, welmv4_inplace_rope_npu_all.csv line 47), i.e. 871 GB/s of the
# same 33,685,504 algorithmic bytes.  vs_baseline = value / this.
PUBLISHED_GBS = 871.0
PUBLISHED_SOURCE = ("reference CSV line 47: prefill_m16384 candidate kernel 38.69 us/launch (NPU event timing, "
                    "Ascend 950PR) = 871 GB/s of the same algorithmic bytes")


def algorithmic_bytes(tokens: int) -> int:
    return 2056 * tokens


def workload_config(world: int) -> dict:
    return {
        "workload": "ordinary prefill in-place partial RoPE, M=16384 tokens per GPU, "
                    "Q bf16 [16384,6,256], K bf16 [16384,1,256], positions 0..16383, "
                    "cos/sin fp32 [16384,64] base 1e4, rope lanes 192..255",
        "tokens_per_gpu": TOKENS,
        "global_tokens": TOKENS * world,
        "head_dim": 256,
        "rope_dim": 64,
        "q_heads": 6,
        "k_heads": 1,
        "parallelism": f"request-sharded dp{world}",
        "l2_policy": f"{BUFFER_SETS} rotating buffer sets (~{BUFFER_SETS * algorithmic_bytes(TOKENS) / 1e6:.0f} MB "
                     "touched between reuses > 126 MB L2)",
        "bytes_per_launch": algorithmic_bytes(TOKENS),
    }


# ---------------------------------------------------------------------------
# Distributed plumbing.
# ---------------------------------------------------------------------------
def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def init_dist(world: int, local_rank: int):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    return dist


def max_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(dist, value: float, device) -> list[float]:
    """Every rank's value, in rank order (after the timed region)."""
    if dist is None:
        return [value]
    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def barrier(dist, device) -> None:
    if dist is not None:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ---------------------------------------------------------------------------
# Peaks and profile figures.
# ---------------------------------------------------------------------------
def hbm_peak() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        value = float(json.loads(path.read_text())["hbm_gbs"])
        return value, "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic() -> tuple[int | None, str]:
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of
    one ncu capture of the bench kernel) as recorded in the committed profile
    summary, and where the figure comes from.  A bench run cannot profile
    itself, so the figure is the last capture's, not this run's."""
    try:
        for line in PROFILE_SUMMARY.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                value = int(float(line.split(":", 1)[1].strip().split()[0]))
                return value, (f"profile summary {PROFILE_SUMMARY.relative_to(REPO)} (ncu dram__bytes_read.sum + "
                               "dram__bytes_write.sum of one launch, captured separately; not measured by this run)")
    except Exception:  # noqa: BLE001
        return None, "no profile summary"
    return None, "no traffic line in the profile summary"


# ---------------------------------------------------------------------------
# CPU leg (the reference's CPU algorithm, via the oracle port).
# ---------------------------------------------------------------------------
def cpu_reference_time(inputs, runs: int, warmup: int = 1) -> tuple[list[float], int]:
    from oracle import rope_oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    times = []
    for i in range(warmup + runs):
        t0 = time.perf_counter()
        rope_oracle.reference_outputs(inputs.query, inputs.key, inputs.positions, None, inputs.cache)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return times, threads


def run_reference_arm(args) -> int:
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from testfiles_b200 import workloads

    case = workloads.Case("bench_prefill_m16384", "prefill", TOKENS, flavour="baseline")
    inputs = workloads.make_inputs(case, "cpu")
    # Each step is a bounded sample of the workload: the first `sample`
    # tokens (a multiple of 64), sized so all warm-up + timed steps take about
    # REFERENCE_BUDGET_S seconds of CPU time.
    full, threads = cpu_reference_time(inputs, runs=1, warmup=1)
    budget = REFERENCE_BUDGET_S / (args.steps + args.warmup)
    sample = int(min(TOKENS, max(64, TOKENS * budget / full[0])) // 64 * 64)
    part = workloads.Inputs(inputs.query[:sample], inputs.key[:sample], inputs.positions[:sample], inputs.cache)
    times, threads = cpu_reference_time(part, runs=args.steps, warmup=max(0, args.warmup))
    per_sample = statistics.mean(times)
    gbs = algorithmic_bytes(sample) / per_sample / 1e9
    # The workload is the GPU arm's at this N: world requests of 16384 tokens
    # (one per GPU there); the CPU path runs them one after another on this
    # host, so a step of the global batch takes world x 16384 / sample times
    # the sample's time, and the rate (GB/s) is the sample's.
    global_tokens = TOKENS * world
    per_step = per_sample * global_tokens / sample
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step * 1e3, 4),
        "us_per_launch": round(per_sample * 1e6 * TOKENS / sample, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(gbs / PUBLISHED_GBS, 4),
        "vs_baseline_source": PUBLISHED_SOURCE,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 Q/K, positions 0..M-1)",
        "config": workload_config(world),
        "cpu_baseline": {
            "value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"first {sample} of the 16384 tokens of one request per step (reference torch CPU path "
                      f"restated), {args.steps} steps after {args.warmup} warm-up, mean; the global batch of "
                      f"{world} request(s) runs at this rate on this host's cores, so ms_per_step is "
                      f"{global_tokens} / {sample} sample times; us_per_launch is one 16384-token request",
        },
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm.
# ---------------------------------------------------------------------------
def timed_steps(step, count: int, dist, device, stream) -> float:
    """Max-over-ranks CUDA-event milliseconds of `count` calls of `step`."""
    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(count):
        step()
    end.record(stream)
    barrier(dist, device)
    return max_over_ranks(dist, start.elapsed_time(end), device)


# ---------------------------------------------------------------------------
# Result checks of the GPU arm: after timing, each leg runs once more on
# pristine inputs; rank 0 gathers every rank's rows (NCCL all_gather when N > 1)
# and compares their SHA-256 with the digest of the reference's own outputs
# for that configuration, recorded by tests/golden/gen_golden.py.
# ---------------------------------------------------------------------------
GOLDEN_OUTPUTS = REPO / "tests" / "golden" / "golden_outputs.json"
L2_BYTES = 126 * 1024 * 1024
MIRROR_CASE = "b_mirror_segmented_n16384_bs128_uneven"
PREFILL_CASE = "b_prefill_m16384"


def sha256_rows(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes, bf16 taken as int16 (the fixtures' rule)."""
    import hashlib

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def golden_outputs(case_name: str) -> dict | None:
    try:
        return json.loads(GOLDEN_OUTPUTS.read_text())["cases"][case_name]["outputs"]
    except Exception:  # noqa: BLE001
        return None


def gather_rows(dist, t: torch.Tensor, counts: list[int]) -> torch.Tensor | None:
    if dist is None:
        return t
    from testfiles_b200 import sharding

    return sharding.gather_rows(t, counts)


def parity_record(dist, rank: int, q: torch.Tensor, k: torch.Tensor, q_counts: list[int], k_counts: list[int],
                  case_name: str, copies: int = 1) -> dict | None:
    """Gathers Q and K rows to rank 0 and compares them with the golden
    digests of `case_name` (`copies` identical requests laid end to end)."""
    q_all = gather_rows(dist, q, q_counts)
    k_all = gather_rows(dist, k, k_counts)
    if rank != 0:
        return None
    want = golden_outputs(case_name)
    if want is None:
        return {"bit_exact": None, "reason": f"no golden digest for {case_name}"}
    ok = True
    for qc, kc in zip(q_all.chunk(copies), k_all.chunk(copies)):
        ok &= sha256_rows(qc) == want["query"] and sha256_rows(kc) == want["key"]
    return {
        "bit_exact": bool(ok),
        # equal digests mean equal bits: no lane differs (0 ulp, lanes 0..191 untouched)
        "max_abs_q": 0.0 if ok else None,
        "max_abs_k": 0.0 if ok else None,
        "max_ulp": 0 if ok else None,
        "rows_checked": {"query": int(q_all.shape[0]), "key": int(k_all.shape[0])},
        "compared_with": f"SHA-256 of the reference's own outputs for {case_name} "
                         f"({GOLDEN_OUTPUTS.relative_to(REPO)}), per request",
        "gathered": "NCCL all_gather to rank 0" if dist is not None else "single rank",
    }


def replay_leg_us(launches: list, dist, device, stream, graph_launches: int = 64,
                  replays: int = 8) -> tuple[float, list[float]]:
    """Max-over-ranks µs per launch of `launches` (one callable per buffer
    set, used in rotation), replayed from a warmed CUDA graph, and every
    rank's own µs per launch in rank order."""
    for f in launches[:3]:
        f()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(graph_launches):
            launches[i % len(launches)]()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist, device)
    torch.cuda._sleep(200_000)
    start.record(stream)
    for _ in range(replays):
        g.replay()
    end.record(stream)
    barrier(dist, device)
    own = start.elapsed_time(end)
    ms = max_over_ranks(dist, own, device)
    ranks = all_ranks(dist, own, device)
    del g
    per = 1e3 / (replays * graph_launches)
    return ms * per, [round(x * per, 3) for x in ranks]


def sets_for(nbytes: int) -> int:
    """Buffer sets so that more than 2 x L2 of algorithmic bytes lie between reuses."""
    return int(min(64, max(2, -(-2 * L2_BYTES // max(nbytes, 1)))))


def strong_prefill_leg(dist, rank: int, world: int, device, stream, peak: float) -> dict:
    """The headline's single M=16384 request split over the ranks in
    64-aligned token ranges (strong scaling): value = its algorithmic bytes
    over the slowest rank's µs per launch."""
    import testfiles_b200 as welm
    from testfiles_b200 import sharding, workloads

    case = workloads.find_case(PREFILL_CASE)
    host = workloads.make_inputs(case, "cpu")
    ranges = [sharding.shard_tokens(TOKENS, world, r) for r in range(world)]
    t0, t1 = ranges[rank]
    local = workloads.Inputs(host.query[t0:t1], host.key[t0:t1], host.positions[t0:t1], host.cache)
    sets = [local.to(device) for _ in range(sets_for(algorithmic_bytes(t1 - t0)))]
    us, rank_us = replay_leg_us([lambda b=b: welm.welmv4_inplace_rope_npu(b.query, b.key, b.positions, b.cache)
                                 for b in sets], dist, device, stream)
    del sets
    fresh = local.to(device)
    welm.welmv4_inplace_rope_npu(fresh.query, fresh.key, fresh.positions, fresh.cache)
    counts = [b - a for a, b in ranges]
    check = parity_record(dist, rank, fresh.query, fresh.key, counts, counts, PREFILL_CASE)
    gbs = algorithmic_bytes(TOKENS) / (us * 1e3)
    return {
        "workload": "ordinary prefill M=16384 (one request) split over the GPUs in 64-aligned token ranges",
        "scaling": "strong", "tokens_per_gpu": counts, "us_per_launch": round(us, 3), "rank_us_per_launch": rank_us,
        "value": round(gbs, 2), "unit": "GB/s", "tokens_per_s": round(TOKENS / (us * 1e-6), 1),
        "frac_of_n_gpu_peak": round(gbs / (peak * world), 4), "parity": check,
    }


def mirror_sharded_leg(dist, rank: int, world: int, device, stream, peak: float) -> dict:
    """The segmented KV mirror N=16384, BS=128 seeded-uneven requests, split
    over the ranks by whole requests balanced by tokens: each rank rotates its
    K rows and its requests' Q rows with last_index rebased to its first token
    and a tile table rebuilt from its own requests.  value = the global
    algorithmic bytes over the slowest rank's µs per launch."""
    import testfiles_b200 as welm
    from testfiles_b200 import sharding, workloads

    case = workloads.find_case(MIRROR_CASE)
    full = workloads.make_inputs(case, "cpu")
    lens = case.segment_lens
    ranges = sharding.shard_requests(lens, world)
    batches = [sharding.local_batch(lens, rr, full.last_index.tolist()) for rr in ranges]
    mine = batches[rank]
    r0, r1 = ranges[rank]

    def local_bytes(b) -> int:
        return 520 * b.n_tokens + 1544 * (b.request_end - b.request_begin) + 4 * len(b.tile_starts)

    local = workloads.Inputs(full.query[r0:r1], full.key[mine.token_begin:mine.token_end],
                             full.positions[mine.token_begin:mine.token_end], full.cache,
                             torch.tensor(mine.last_index, dtype=torch.int64),
                             torch.tensor(mine.tile_starts, dtype=torch.int32), mine.num_work_tiles, 1)
    sets = [local.to(device) for _ in range(sets_for(local_bytes(mine)))]

    def call(b) -> None:
        welm.welmv4_inplace_rope_npu(b.query, b.key, b.positions, b.cache, b.last_index, b.segment_tile_starts)

    us, rank_us = replay_leg_us([lambda b=b: call(b) for b in sets], dist, device, stream)
    del sets
    fresh = local.to(device)
    call(fresh)
    check = parity_record(dist, rank, fresh.query, fresh.key, [r[1] - r[0] for r in ranges],
                          [b.n_tokens for b in batches], MIRROR_CASE)
    total = sum(local_bytes(b) for b in batches)
    gbs = total / (us * 1e3)
    return {
        "workload": "segmented KV mirror N=16384, BS=128 seeded-uneven requests, split over the GPUs by whole "
                    "requests (rebased last_index, tile tables rebuilt per GPU)",
        "scaling": "strong", "requests_per_gpu": [r[1] - r[0] for r in ranges],
        "tokens_per_gpu": [b.n_tokens for b in batches], "bytes_per_launch": total,
        "us_per_launch": round(us, 3), "rank_us_per_launch": rank_us, "value": round(gbs, 2), "unit": "GB/s",
        "tokens_per_s": round(16384 / (us * 1e-6), 1), "frac_of_n_gpu_peak": round(gbs / (peak * world), 4),
        "frac_of_peak_n1_equivalent": round(gbs / peak, 4), "parity": check,
    }


def host_copy_ceiling(h2d: int, d2h: int, steps: int, dist, device, stream, h_q, h_k, h_p) -> dict:
    """Two ceilings for the e2e step's bus traffic, each with the two
    directions on two streams at once and on every rank at the same time (max
    over ranks):

    * contiguous: h2d bytes from one pinned host buffer to the device and d2h
      bytes back (the link's bulk rate, whatever the layout);
    * strided: the same rope-lane slices the e2e step moves, in the caller's
      layout (128-byte pieces 512 bytes apart), by 2-D DMA copies through the
      library's welm_rope_copy_rope_lanes: pinned Q/K lanes and positions to
      device buffers, and device lanes back to pinned buffers."""
    from testfiles_b200 import host as welm_host

    side = torch.cuda.Stream(device)

    def both_ways(to_device, to_host):
        def step() -> None:
            side.wait_stream(stream)
            to_device(stream)
            with torch.cuda.stream(side):
                to_host(side)
            stream.wait_stream(side)
        return step

    src_h = torch.empty(h2d, dtype=torch.uint8).pin_memory()
    dst_d = torch.empty(h2d, dtype=torch.uint8, device=device)
    src_d = torch.empty(d2h, dtype=torch.uint8, device=device)
    dst_h = torch.empty(d2h, dtype=torch.uint8).pin_memory()
    contiguous = both_ways(lambda st: dst_d.copy_(src_h, non_blocking=True),
                           lambda st: dst_h.copy_(src_d, non_blocking=True))
    us_c = timed_steps(contiguous, steps, dist, device, stream) * 1e3 / steps

    d_q, d_k, d_p = (torch.empty_like(h_q, device=device), torch.empty_like(h_k, device=device),
                     torch.empty_like(h_p, device=device))
    o_q, o_k = torch.empty_like(h_q).pin_memory(), torch.empty_like(h_k).pin_memory()
    rows = h_q.shape[0]

    def lanes_in(st) -> None:
        welm_host._copy_lanes(d_q, h_q, rows, 6, 0, st)
        welm_host._copy_lanes(d_k, h_k, rows, 1, 0, st)
        d_p.copy_(h_p, non_blocking=True)

    def lanes_out(st) -> None:
        welm_host._copy_lanes(o_q, d_q, rows, 6, 1, st)
        welm_host._copy_lanes(o_k, d_k, rows, 1, 1, st)

    us_s = timed_steps(both_ways(lanes_in, lanes_out), steps, dist, device, stream) * 1e3 / steps
    return {"us_per_step": round(us_c, 2), "h2d_gb_s": round(h2d / (us_c * 1e3), 2),
            "d2h_gb_s": round(d2h / (us_c * 1e3), 2),
            "how": "contiguous pinned host -> device and device -> pinned host copies of the e2e step's bytes, "
                   "both directions at once, every rank at once",
            "strided_us_per_step": round(us_s, 2),
            "strided_how": "the same rope-lane slices in the caller's layout (128-byte pieces, 512 bytes apart) by "
                           "2-D DMA copies (welm_rope_copy_rope_lanes), both directions at once, every rank at once"}


# One configuration of each other benchmark family, timed after the headline
# (rank 0, N=1) with the launcher's method: graph replay over L2-cold buffer
# sets, plus a same-size device copy as the practical ceiling.
OTHER_CONFIGS = ("b_prefill_m8192", "b_decode_m1", "b_decode_m128", "b_mirror_contiguous_n16384",
                 "b_mirror_segmented_n16384_bs128_uneven")


def other_config_records(device) -> list[dict]:
    from testfiles_b200 import launcher, workloads

    keep = ("case", "phase", "n_tokens", "batch_size", "us_per_launch", "gb_s", "hbm_frac", "same_size_copy_us",
            "frac_of_same_size_copy", "l2_cold")
    # each configuration is timed three times and the fastest record kept:
    # single timings after the headline's legs can read high
    def best(timer):
        return min((timer() for _ in range(3)), key=lambda rec: rec["us_per_launch"])

    out = []
    for name in OTHER_CONFIGS:
        rec = best(lambda: launcher.time_case(workloads.find_case(name), device, copy_ceiling=True))
        out.append({k: rec[k] for k in keep})
    # the KV mirror fused with the paged KV-cache write (random slots)
    rec = best(lambda: launcher.time_kv_write(16384, 128, device))
    out.append({k: rec.get(k) for k in keep})
    return out


def run_b200_arm(args) -> int:
    import testfiles_b200 as welm
    from testfiles_b200 import host as welm_host
    from testfiles_b200 import launcher, sharding, workloads

    rank, world, local_rank = dist_env()
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = init_dist(world, local_rank)

    # Weak scaling: the global batch is one 16384-token request per rank,
    # sharded by whole requests (no exchange on the hot path).
    shards = sharding.shard_requests([TOKENS] * world, world)
    r0, r1 = shards[rank]
    local = sharding.local_batch([TOKENS] * world, (r0, r1))
    n_tokens = local.n_tokens
    assert n_tokens == TOKENS

    case = workloads.Case("bench_prefill_m16384", "prefill", n_tokens, flavour="baseline")
    host = workloads.make_inputs(case, "cpu")
    cache = host.cache.to(device)
    positions = host.positions.to(device)
    sets = []
    for _ in range(BUFFER_SETS):
        sets.append((host.query.to(device), host.key.to(device), positions.clone(), cache.clone()))
    launches = 0

    def step(i: int) -> None:
        q, k, p, c = sets[i % BUFFER_SETS]
        welm.welmv4_inplace_rope_npu(q, k, p, c)

    stream = torch.cuda.current_stream(device)
    sampler = ClockSampler(device.index)
    with sampler:
        # Eager warm-up (also loads the kernels before any capture).
        for i in range(max(3, args.warmup)):
            step(i)
        torch.cuda.synchronize(device)

        # Capture the timed launches: `body` holds GRAPH_LAUNCHES launches
        # cycling through the buffer sets, `tail` the remainder, so exactly
        # K launches run in the timed region.  Every graph that the timed
        # region replays is itself replayed three times first, so no first
        # replay (graph upload, cold instruction caches) is timed.
        def capture(count: int):
            if count == 0:
                return None
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(count):
                    step(i)
            return g

        reps, rem = divmod(args.steps, GRAPH_LAUNCHES)
        body = capture(GRAPH_LAUNCHES) if reps else None
        tail = capture(rem)
        for _ in range(3):
            for g in (body, tail):
                if g is not None:
                    g.replay()
        torch.cuda.synchronize(device)

        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(dist, device)
        # ~100 us of device-side delay ahead of the start event, so the host
        # has submitted the graphs before timing begins (a short timed region
        # would otherwise include the submission latency); the first timed
        # launch still starts cold, with no previous launch of the op to
        # overlap with
        torch.cuda._sleep(200_000)
        start.record(stream)
        for _ in range(reps):
            body.replay()  # reps > 0 only when body was captured
        if tail is not None:
            tail.replay()
        end.record(stream)
        barrier(dist, device)
        launches += args.steps
        own_ms = start.elapsed_time(end)
        elapsed_ms = max_over_ranks(dist, own_ms, device)
        rank_ms = all_ranks(dist, own_ms, device)

    # Every device-only leg runs before the host-memory legs: in one process,
    # device launches timed after the staged host transport had run measured
    # up to 20 % slower (prefill M=8192 3.50 -> 4.19 us; the strong-scaled
    # M=8192 half 3.5 -> 4.3), so the e2e legs come last.  `clocks` covers the
    # headline only; everything after it gets its own sampler (`clocks_legs`).
    del body, tail
    with ClockSampler(device.index) as legs_sampler:
        # One configuration of each other family (one GPU only).
        others = other_config_records(device) if world == 1 and not args.no_config_sweep else None

        # Same-size copy ceiling: a plain device copy moving the same number of
        # bytes per step (half read, half written), replayed and timed exactly
        # like the op, over rotating buffers larger than L2.
        half = algorithmic_bytes(TOKENS) // 2 // 4096 * 4096  # 4 KiB multiple: the copy's fast path
        pairs = [(torch.empty(half, dtype=torch.uint8, device=device).fill_(1),
                  torch.empty(half, dtype=torch.uint8, device=device)) for _ in range(BUFFER_SETS)]
        copy_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(copy_graph):
            for i in range(GRAPH_LAUNCHES):
                src, dst = pairs[i % BUFFER_SETS]
                dst.copy_(src)
        copy_ms = timed_steps(copy_graph.replay, 20, dist, device, stream) / (20 * GRAPH_LAUNCHES)
        del copy_graph, pairs
        # Two tighter ceilings, each rank on its own (no collective): the same
        # bytes through the library's streaming copy kernel launched like the
        # op, and the op's own loads and stores over its buffers without the
        # position / cos-sin gather and the arithmetic.
        stream_copy_us = launcher.stream_copy_us(algorithmic_bytes(TOKENS), BUFFER_SETS, device, graph_launches=64)
        slice_floor_us = launcher.slice_floor_us([(q, k) for q, k, _, _ in sets], device, graph_launches=64)
        torch.cuda.synchronize(device)
        del sets
        torch.cuda.empty_cache()

        peak, peak_kind = hbm_peak()
        # The headline's result on pristine inputs, gathered and checked; then
        # the strong-scaling split of the same request and the request-sharded
        # segmented KV mirror, each timed and checked the same way.  Every rank
        # takes every step (each holds collectives).
        fresh = host.to(device)
        welm.welmv4_inplace_rope_npu(fresh.query, fresh.key, fresh.positions, fresh.cache)
        headline_parity = parity_record(dist, rank, fresh.query, fresh.key, [TOKENS] * world, [TOKENS] * world,
                                        PREFILL_CASE, copies=world)
        del fresh
        strong = strong_prefill_leg(dist, rank, world, device, stream, peak)
        mirror = mirror_sharded_leg(dist, rank, world, device, stream, peak)
        torch.cuda.empty_cache()

        # End to end through the public host-memory API: Q, K and positions
        # start in pinned host memory every step and the rotated Q and K end
        # there (only the rotated lanes cross PCIe).
        e2e_steps = max(1, min(args.steps, args.e2e_steps))
        h_q = host.query.pin_memory()
        h_k = host.key.pin_memory()
        h_p = host.positions.pin_memory()

        def e2e_step() -> None:
            welm_host.welmv4_inplace_rope_host(h_q, h_k, h_p, cache)  # pinned: the mapped transport

        e2e_ms = timed_steps(e2e_step, e2e_steps, dist, device, stream)
        launches_e2e = e2e_steps

        def staged_step() -> None:
            welm_host.welmv4_inplace_rope_host(h_q, h_k, h_p, cache, transport="staged")

        staged_ms = timed_steps(staged_step, e2e_steps, dist, device, stream)

        # The same through whole-tensor copies (what a caller without the
        # host API would do), reported beside it.
        d_q, d_k, d_p = torch.empty_like(h_q, device=device), torch.empty_like(h_k, device=device), \
            torch.empty_like(positions)

        def full_copy_step() -> None:
            d_q.copy_(h_q, non_blocking=True)
            d_k.copy_(h_k, non_blocking=True)
            d_p.copy_(h_p, non_blocking=True)
            welm.welmv4_inplace_rope_npu(d_q, d_k, d_p, cache)
            h_q.copy_(d_q, non_blocking=True)
            h_k.copy_(d_k, non_blocking=True)

        full_ms = timed_steps(full_copy_step, e2e_steps, dist, device, stream)
        del d_q, d_k, d_p
        # the plain host-copy ceilings of the e2e step
        h2d_bytes, d2h_bytes = welm_host.lane_bytes(TOKENS)
        host_ceiling = host_copy_ceiling(h2d_bytes, d2h_bytes, e2e_steps, dist, device, stream, h_q, h_k, h_p)
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()

    per_step_s = elapsed_ms / 1e3 / args.steps
    total_bytes = algorithmic_bytes(TOKENS) * world
    value = total_bytes / per_step_s / 1e9
    per_launch_gbs = algorithmic_bytes(TOKENS) / per_step_s / 1e9
    e2e_per_step = e2e_ms / 1e3 / e2e_steps
    full_per_step = full_ms / 1e3 / e2e_steps
    staged_per_step = staged_ms / 1e3 / e2e_steps
    h2d, d2h = welm_host.lane_bytes(TOKENS)
    traffic, traffic_source = profiled_traffic()

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            times, threads = cpu_reference_time(host, runs=5)
            cpu_t = statistics.median(times)
            cpu = {
                "value": round(algorithmic_bytes(TOKENS) / cpu_t / 1e9, 3),
                "unit": "GB/s",
                "cores": threads,
                "kind": "port",
                "sample": "full M=16384 prefill (reference torch CPU path restated), median of 5 after 1 warm-up; "
                          f"{cpu_t * 1e3:.2f} ms/launch",
            }
        line = {
            "impl": "b200",
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(per_step_s * 1e3, 6),
            "us_per_launch": round(per_step_s * 1e6, 3),
            "rank_us_per_launch": [round(ms * 1e3 / args.steps, 3) for ms in rank_ms],
            "tokens_per_s": round(TOKENS * world / per_step_s, 1),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / PUBLISHED_GBS, 4),
            "vs_baseline_source": PUBLISHED_SOURCE,
            "dtype": "bf16",
            "math": "f32 (separate mul/sub/add roundings, one RNE to bf16)",
            "data": "synthetic (seeded N(0,1) bf16 Q/K, positions 0..M-1)",
            "config": workload_config(world),
            "parity": headline_parity,
            "roofline": {
                "bound": "hbm",
                "achieved": round(per_launch_gbs, 2),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(per_launch_gbs / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "frac_of_8tbs_spec": round(per_launch_gbs / 8000.0, 4),
                "traffic": traffic,
                "traffic_source": traffic_source,
                "same_size_copy_us": round(copy_ms * 1e3, 3),
                "frac_of_same_size_copy": round(copy_ms * 1e3 / (per_step_s * 1e6), 4),
                "same_size_copy": "torch copy_ of 16.8 MB (33.7 MB of traffic) per step, graph-replayed over "
                                  "8 rotating buffer pairs like the op: the practical ceiling at this size",
                "stream_copy_us": round(stream_copy_us, 3),
                "frac_of_stream_copy": round(stream_copy_us / (per_step_s * 1e6), 4),
                "stream_copy": "the library's streaming copy kernel (welm_rope_ceiling_copy, PDL) on the same "
                               "bytes and buffer rotation: one 16-byte vector per thread up to a full-occupancy "
                               "wave, four per thread above (this size is above)",
                "slice_floor_us": round(slice_floor_us, 3),
                "frac_of_slice_floor": round(slice_floor_us / (per_step_s * 1e6), 4),
                "slice_floor": "welm_rope_ceiling_slices on the op's own buffers: the same launch shape, loads "
                               "and stores of the rope slices, without the position / cos-sin gather and "
                               "the arithmetic",
                "kernel": "rope_ordinary_stream_kernel<vec=1> (one item per thread, pre-wait L2 prefetch)",
                "bytes_per_launch": algorithmic_bytes(TOKENS),
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": round(total_bytes / e2e_per_step / 1e9, 3),
                "unit": "GB/s",
                "us_per_step": round(e2e_per_step * 1e6, 2),
                "steps": e2e_steps,
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "host_ceiling": host_ceiling,
                "frac_of_host_ceiling": round(host_ceiling["us_per_step"] / (e2e_per_step * 1e6), 4),
                "frac_of_strided_host_ceiling": round(host_ceiling["strided_us_per_step"] / (e2e_per_step * 1e6), 4),
                "api": "testfiles_b200.welmv4_inplace_rope_host (pinned host Q/K/positions, mapped transport: "
                       "one kernel reads each 128-byte rope slice from host memory over PCIe and writes it back; "
                       "every transfer in the timed region)",
                "staged_copies": {
                    "value": round(total_bytes / staged_per_step / 1e9, 3),
                    "us_per_step": round(staged_per_step * 1e6, 2),
                    "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": "welmv4_inplace_rope_host(transport='staged'): rope-lane copies in and out, "
                           "2048-token chunks pipelined over 3 streams",
                },
                "whole_tensor_copies": {
                    "value": round(total_bytes / full_per_step / 1e9, 3),
                    "us_per_step": round(full_per_step * 1e6, 2),
                    "h2d_bytes_per_step": host.query.numel() * 2 + host.key.numel() * 2 + host.positions.numel() * 8,
                    "d2h_bytes_per_step": host.query.numel() * 2 + host.key.numel() * 2,
                    "api": "welmv4_inplace_rope_npu on device copies of the whole pinned tensors",
                },
            },
            "strong_scaling": strong,
            "mirror_sharded": mirror,
            "clocks": sampler.summary(),
            "clocks_legs": legs_sampler.summary(),
            "gpu_launches": launches,
            "other_configs": others,
            "gpu_launches_e2e": launches_e2e,
        }
    if dist is not None:
        dist.barrier(device_ids=[device.index])
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20000)
    parser.add_argument("--warmup", type=int, default=50)
    parser.add_argument("--e2e-steps", type=int, default=100)
    parser.add_argument("--no-config-sweep", action="store_true",
                        help="skip the one-per-family timing of the other benchmark configurations")
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    args = parser.parse_args()
    if args.steps <= 0:
        raise SystemExit("--steps must be positive")
    if args.impl == "reference":
        return run_reference_arm(args)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the op has no CPU path)")
    return run_b200_arm(args)


if __name__ == "__main__":
    raise SystemExit(main())
