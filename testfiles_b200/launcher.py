"""Launch / time any catalogue case of the in-place RoPE (profiling launcher).

    python -m testfiles_b200.launcher --cases b_mirror_segmented_n16384_bs128_uneven --iters 20
    python -m testfiles_b200.launcher --cases baseline --time --json times.jsonl
    python -m testfiles_b200.launcher --cases b_prefill_m16384 --host mapped

``--iters N`` launches the op N times eagerly on one buffer set with a fixed
kernel name per path (``rope_ordinary_head_kernel`` for dense launches of at
most 3328 tokens, ``rope_ordinary_stream_kernel`` for larger dense launches
and segmented ones whose tiles are mostly full, ``rope_ordinary_kernel`` for
other segmented ones; ``rope_mirror_head_kernel``), for
``ncu -k regex:…`` captures — the B200 analogue of the reference's msprof
launch stub (run_welmv4_inplace_rope_prod_m16384_npu.py:1-60).

``--time`` measures each case the way ``bench.py`` measures its headline:
launches replayed from a CUDA graph over rotating buffer sets (enough sets
that more than 2 x 126 MB of algorithmic bytes are touched between reuses,
capped at 64 sets; smaller cases therefore run partly from L2, which the
record states), CUDA events on the launching stream, median of 5 trials.
Each record is one JSON line whose fields follow the reference's CSV record
(bench_welmv4_inplace_rope_npu.py:1143-1162,1529-1540): ``record_type``,
case fields, then µs per launch, tokens/s, GB/s of algorithmic bytes and the
fraction of the HBM peak, plus the SM clock and throttle reasons sampled
during the timed replays; ``--csv`` writes the records as one table.
``--copy-ceiling`` adds the time of a plain device
copy moving the same bytes (half read, half written), replayed and rotated
exactly like the op: the practical ceiling at that size, where launch and
pipeline-fill costs weigh as much as bandwidth.  It gives two copies: the
runtime's device copy (``same_size_copy_us``) and the library's streaming
copy kernel, launched like the op (``stream_copy_us``).  Ordinary cases also
get ``slice_floor_us``: the op's own loads and stores without its gather
and arithmetic, over the same buffers.

``--gather-only`` (with ``--iters``) launches only the op's position and
cos/sin gather (``ceiling_gather_kernel``) on the case's positions, so an ncu
capture of it gives the gather's L2 hit rate apart from the Q/K slices.
``--host mapped|staged`` times the host-memory entry instead (ordinary
cases): Q, K and positions in pinned host memory, every PCIe transfer inside
the timed region, µs per call and GB/s each way over the bus.
``--kv-write N,BS`` times the fused KV-mirror cache write (with ``--time``;
with ``--iters`` it only launches it, for ncu).  ``--fused-qkv M`` times
prefill on strided Q/K views of a fused QKV projection output beside a
contiguous Q copy followed by the op.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import sys
from typing import Iterable, Optional

import torch

from . import _native, ops, workloads
from .clocks import ClockSampler

L2_BYTES = 126 * 1024 * 1024
SPEC_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def measured_hbm_peak() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def case_fields(case: workloads.Case) -> dict:
    return {
        "case": case.name,
        "phase": case.phase,
        "flavour": case.flavour,
        "path": "kv_mirror" if case.is_mirror else "normal",
        "n_tokens": case.n_tokens,
        "q_rows": case.q_rows,
        "batch_size": case.batch_size,
        "request_count": len(case.segment_lens),
        "has_segments": int(case.is_segmented),
        "segment_lens": "|".join(str(x) for x in case.segment_lens) if len(case.segment_lens) <= 16 else
        f"{len(case.segment_lens)} requests",
    }


def select_cases(spec: str) -> list[workloads.Case]:
    ref = workloads.reference_cases()
    base = workloads.baseline_cases()
    groups = {
        "reference": ref,
        "baseline": base,
        "decode": [c for c in base if c.phase == "decode"],
        "prefill": [c for c in base if c.phase == "prefill"],
        "mirror": [c for c in base if c.is_mirror],
        "segmented": [c for c in ref if c.phase == "segmented_prefill"],
    }
    out: list[workloads.Case] = []
    for item in spec.split(","):
        item = item.strip()
        if not item:
            continue
        out.extend(groups[item] if item in groups else [workloads.find_case(item)])
    return out


def _launch(inp: workloads.Inputs) -> None:
    lens = inp.extra.get("seq_lens")
    if lens is not None:  # segmented KV mirror straight from request lengths
        ops.rope_mirror_from_lens(inp.query, inp.key, inp.positions, inp.cache, lens)
        return
    ops.welmv4_inplace_rope_npu(inp.query, inp.key, inp.positions, inp.cache, inp.last_index,
                                inp.segment_tile_starts)


def _with_lens(case: workloads.Case, inp: workloads.Inputs, device: torch.device) -> workloads.Inputs:
    if case.is_mirror and case.is_segmented:
        inp.extra["seq_lens"] = torch.tensor(case.segment_lens, dtype=torch.int64, device=device)
    return inp


def _replay_us(graph: "torch.cuda.CUDAGraph", device: torch.device, trials: int, replays: int,
               graph_launches: int) -> float:
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    samples = []
    for _ in range(trials):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(replays):
            graph.replay()
        end.record(stream)
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1e3 / (replays * graph_launches))
    return statistics.median(samples)


def same_size_copy_us(nbytes: int, sets: int, device: torch.device, trials: int = 5, graph_launches: int = 64,
                      replays: int = 20) -> float:
    """µs per device copy of about ``nbytes // 2`` bytes (``nbytes`` of
    traffic), graph-replayed over ``sets`` rotating source/destination pairs.
    The size is rounded DOWN to a multiple of 4 KiB: device copies of other
    sizes take a markedly slower path (M=8191's 8.4 MB copy: 7.4 µs against
    4.2 µs for M=8192's), and rounding down keeps the ceiling on the copy's
    side."""
    half = max(4096, nbytes // 2 // 4096 * 4096)
    pairs = [(torch.ones(half, dtype=torch.uint8, device=device), torch.empty(half, dtype=torch.uint8, device=device))
             for _ in range(sets)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            src, dst = pairs[i % sets]
            dst.copy_(src)
    us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph, pairs
    return us


def ceiling_copy(dst: torch.Tensor, src: torch.Tensor, nbytes: int) -> None:
    """The library's streaming copy (welm_rope_ceiling_copy) of ``nbytes``
    (a multiple of 16) from ``src`` to ``dst``, both CUDA, on the current
    stream of their device."""
    if src.device != dst.device or src.device.type != "cuda":
        raise ValueError("ceiling_copy needs two tensors on one CUDA device")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise ValueError("ceiling_copy needs contiguous tensors")
    if nbytes < 0 or nbytes > min(src.numel() * src.element_size(), dst.numel() * dst.element_size()):
        raise ValueError("nbytes exceeds a buffer")
    lib = _native.load()
    rc = ops._call(dst.device, lib.welm_rope_ceiling_copy, dst.data_ptr(), src.data_ptr(), int(nbytes),
                   torch.cuda.current_stream(dst.device).cuda_stream)
    _native.check("welm_rope_ceiling_copy", rc)


def ceiling_slices(q: torch.Tensor, k: torch.Tensor) -> None:
    """The ordinary kernel's loads and stores alone (welm_rope_ceiling_slices):
    the rope slices of every row of ``q`` [M, 6, 256] and ``k`` [M, 1, 256]
    read and written back unchanged, on the current stream of their device."""
    ops._check_heads(q, "query", ops.NUM_Q_HEADS)
    ops._check_heads(k, "key", ops.NUM_K_HEADS)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise TypeError("ceiling_slices needs bf16 q and k")
    if q.device != k.device or q.device.type != "cuda" or q.shape[0] != k.shape[0]:
        raise ValueError("ceiling_slices needs q and k with the same rows on one CUDA device")
    lib = _native.load()
    rc = ops._call(q.device, lib.welm_rope_ceiling_slices, q.data_ptr(), k.data_ptr(), int(q.shape[0]),
                   int(q.stride(0)), int(k.stride(0)), torch.cuda.current_stream(q.device).cuda_stream)
    _native.check("welm_rope_ceiling_slices", rc)


def ceiling_tma_slices(q: torch.Tensor, k: torch.Tensor, ctas: int = 0, stages: int = 6,
                       status: Optional[torch.Tensor] = None) -> None:
    """The same slices as :func:`ceiling_slices` moved through shared memory
    by TMA (welm_rope_ceiling_tma_slices): ``ctas`` persistent CTAs (0: two
    per SM), a ring of ``stages`` 16-token tiles each, data unchanged."""
    ops._check_heads(q, "query", ops.NUM_Q_HEADS)
    ops._check_heads(k, "key", ops.NUM_K_HEADS)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise TypeError("ceiling_tma_slices needs bf16 q and k")
    if q.device != k.device or q.device.type != "cuda" or q.shape[0] != k.shape[0]:
        raise ValueError("ceiling_tma_slices needs q and k with the same rows on one CUDA device")
    lib = _native.load()
    rc = ops._call(q.device, lib.welm_rope_ceiling_tma_slices, q.data_ptr(), k.data_ptr(), int(q.shape[0]),
                   int(q.stride(0)), int(k.stride(0)), int(ctas), int(stages), ops._status_ptr(status, q.device),
                   torch.cuda.current_stream(q.device).cuda_stream)
    _native.check("welm_rope_ceiling_tma_slices", rc)


def ceiling_gather(positions: torch.Tensor, cache: torch.Tensor) -> None:
    """The ordinary kernels' position and cos/sin gather alone
    (welm_rope_ceiling_gather) over ``positions``, on the current stream of
    their device: for profiling the gather's L2 and DRAM traffic apart from
    the Q/K slices."""
    if positions.device != cache.device or positions.device.type != "cuda":
        raise ValueError("ceiling_gather needs positions and cache on one CUDA device")
    if positions.dtype != torch.int64 or cache.dtype != torch.float32 or cache.dim() != 2 or cache.shape[1] != 64:
        raise TypeError("ceiling_gather needs int64 positions and a float32 [P, 64] cache")
    if not (positions.is_contiguous() and cache.is_contiguous()):
        raise ValueError("ceiling_gather needs contiguous tensors")
    lib = _native.load()
    rc = ops._call(positions.device, lib.welm_rope_ceiling_gather, positions.data_ptr(), cache.data_ptr(),
                   int(positions.numel()), int(cache.shape[0]), None,
                   torch.cuda.current_stream(positions.device).cuda_stream)
    _native.check("welm_rope_ceiling_gather", rc)


def stream_copy_us(nbytes: int, sets: int, device: torch.device, trials: int = 5, graph_launches: int = 64,
                   replays: int = 20) -> float:
    """µs per streaming copy (welm_rope_ceiling_copy) of ``nbytes // 2`` bytes
    rounded down to 16 (``nbytes`` of traffic), graph-replayed over ``sets``
    rotating source/destination pairs like :func:`same_size_copy_us`."""
    half = max(16, nbytes // 2 // 16 * 16)
    pairs = [(torch.ones(half, dtype=torch.uint8, device=device), torch.empty(half, dtype=torch.uint8, device=device))
             for _ in range(sets)]
    ceiling_copy(pairs[0][1], pairs[0][0], half)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            src, dst = pairs[i % sets]
            ceiling_copy(dst, src, half)
    us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph, pairs
    return us


def slice_floor_us(buffers: list[tuple[torch.Tensor, torch.Tensor]], device: torch.device, trials: int = 5,
                   graph_launches: int = 64, replays: int = 20) -> float:
    """µs per welm_rope_ceiling_slices launch over the (q, k) pairs of
    ``buffers`` in rotation: the access-pattern floor of an ordinary launch."""
    ceiling_slices(*buffers[0])
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            ceiling_slices(*buffers[i % len(buffers)])
    us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph
    return us


def tma_floor_us(buffers: list[tuple[torch.Tensor, torch.Tensor]], device: torch.device, stages: int = 6,
                 ctas: int = 0, trials: int = 5, graph_launches: int = 64, replays: int = 20) -> float:
    """µs per welm_rope_ceiling_tma_slices launch over the (q, k) pairs of
    ``buffers`` in rotation, timed like :func:`slice_floor_us`; raises if a
    barrier wait gave up."""
    status = torch.zeros(1, dtype=torch.int32, device=device)
    ceiling_tma_slices(*buffers[0], ctas, stages, status)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            ceiling_tma_slices(*buffers[i % len(buffers)], ctas, stages, status)
    us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph
    if int(status.item()) != 0:
        raise RuntimeError(f"welm_rope_ceiling_tma_slices reported device status {int(status.item())}")
    return us


def time_case(case: workloads.Case, device: torch.device, trials: int = 5, graph_launches: int = 64,
              replays: Optional[int] = None, from_lens: bool = False, copy_ceiling: bool = False,
              shared_cache: bool = False, sets: Optional[int] = None, tma_floor: bool = False) -> dict:
    """µs per launch of ``case`` (graph-replayed over rotating buffer sets);
    ``from_lens`` runs segmented mirror cases through rope_mirror_from_lens.
    ``shared_cache`` gives every set the same cos/sin cache (hot in L2, as
    in serving) instead of a private copy each.  ``sets`` overrides the
    number of buffer sets (default: enough that more than twice the L2
    lies between reuses, at most 64); one or two keep the data L2-resident.
    ``tma_floor`` (dense ordinary cases) also times the TMA-staged slice
    mover on the same buffers, best of 2, 4 and 6 stages."""
    host = workloads.make_inputs(case, "cpu")
    nbytes = workloads.min_bytes(case)
    if sets is None:
        sets = int(min(64, max(2, -(-2 * L2_BYTES // max(nbytes, 1)))))
    elif sets < 1:
        raise ValueError("sets must be at least 1")
    buffers = []
    base = host.to(device)
    for _ in range(sets):
        b = base.clone()
        b.positions = base.positions.clone()
        b.cache = base.cache if shared_cache else base.cache.clone()
        if from_lens:
            _with_lens(case, b, device)
        buffers.append(b)
    for i in range(3):
        _launch(buffers[i % sets])
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            _launch(buffers[i % sets])
    if replays is None:  # about 5 ms of launches per trial
        est_us = 1.5 + nbytes / 5e6
        replays = max(5, min(200, int(5e3 / (est_us * graph_launches))))
    with ClockSampler(device.index) as clocks:
        us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph
    ceiling = {}
    if copy_ceiling and not case.is_mirror and not case.is_segmented:
        floor_us = slice_floor_us([(b.query, b.key) for b in buffers], device, trials, graph_launches, replays)
        ceiling = {"slice_floor_us": round(floor_us, 3), "frac_of_slice_floor": round(floor_us / us, 4)}
    if tma_floor and not case.is_mirror and not case.is_segmented:
        tma = {f"{st}_stages": round(tma_floor_us([(b.query, b.key) for b in buffers], device, st, 0, trials,
                                                  graph_launches, replays), 3) for st in (2, 4, 6)}
        ceiling.update({"tma_slice_floor_us": min(tma.values()), "tma_slice_floor_by_stages": tma})
    del buffers
    peak, kind = measured_hbm_peak()
    gbs = nbytes / (us * 1e3)
    if copy_ceiling:
        copy_us = same_size_copy_us(nbytes, sets, device, trials, graph_launches, replays)
        stream_us = stream_copy_us(nbytes, sets, device, trials, graph_launches, replays)
        ceiling.update({"same_size_copy_us": round(copy_us, 3), "frac_of_same_size_copy": round(copy_us / us, 4),
                        "stream_copy_us": round(stream_us, 3), "frac_of_stream_copy": round(stream_us / us, 4)})
    return {
        "record_type": "timing",
        **case_fields(case),
        "us_per_launch": round(us, 3),
        "tokens_per_s": round(case.n_tokens / (us * 1e-6), 1),
        "bytes_per_launch": nbytes,
        "gb_s": round(gbs, 1),
        "hbm_frac": round(gbs / peak, 4),
        "hbm_peak_gbs": peak,
        "hbm_peak_source": kind,
        "hbm_frac_of_8tbs_spec": round(gbs / SPEC_HBM_GBS, 4),
        **ceiling,
        "clocks": clocks.summary(),
        "buffer_sets": sets,
        "l2_cold": bool(sets * nbytes > 2 * L2_BYTES),
        "cos_sin_cache": "shared by all sets" if shared_cache else "one copy per set",
        "pdl": os.environ.get("WELM_ROPE_PDL", "1") != "0",
        "entry": "rope_mirror_from_lens" if from_lens and case.is_mirror and case.is_segmented
        else "welmv4_inplace_rope_npu",
        "device_name": torch.cuda.get_device_name(device),
        "torch_version": torch.__version__,
        "python_version": platform.python_version(),
    }


def time_host_case(case: workloads.Case, device: torch.device, transport: str, trials: int = 5,
                   calls: int = 20) -> dict:
    """µs per call of the host-memory entry (``welmv4_inplace_rope_host``)
    on pinned host Q/K/positions for an ordinary case, every transfer
    inside the timed region (CUDA events on the current stream)."""
    from . import host as welm_host

    if case.is_mirror:
        raise ValueError("the host-memory entry serves ordinary prefill / decode cases")
    inp = workloads.make_inputs(case, "cpu")
    q, k, pos = inp.query.pin_memory(), inp.key.pin_memory(), inp.positions.pin_memory()
    cache = inp.cache.to(device)
    for _ in range(3):
        welm_host.welmv4_inplace_rope_host(q, k, pos, cache, transport=transport)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    samples = []
    for _ in range(trials):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(calls):
            welm_host.welmv4_inplace_rope_host(q, k, pos, cache, transport=transport)
        end.record(stream)
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1e3 / calls)
    us = statistics.median(samples)
    h2d, d2h = welm_host.lane_bytes(case.n_tokens)
    return {
        "record_type": "host_timing",
        **case_fields(case),
        "transport": transport,
        "us_per_call": round(us, 2),
        "tokens_per_s": round(case.n_tokens / (us * 1e-6), 1),
        "h2d_bytes_per_call": h2d,
        "d2h_bytes_per_call": d2h,
        "pcie_gb_s_each_way": round(d2h / (us * 1e3), 2),
        "gb_s_algorithmic": round(workloads.min_bytes(case) / (us * 1e3), 2),
        "device_name": torch.cuda.get_device_name(device),
    }


def kv_write_bytes(n_tokens: int, batch: int) -> int:
    """Algorithmic bytes of one fused KV-mirror write: per token K and V read
    and written to the cache (4 x 512), position and slot (16), cos/sin row
    (256); per request the Q row read and written (2 x 3072) and last_index."""
    return 2320 * n_tokens + 6152 * batch


def time_kv_write(n_tokens: int, batch: int, device: torch.device, trials: int = 7, graph_launches: int = 64,
                  replays: int = 20, sets: int = 16, iters: int = 0) -> dict:
    """µs per launch of rope_mirror_kv_write on a fused QKV projection output
    [N, 8, 256] with seeded-uneven requests (positions restarting per
    request), random slots of a [300, 64, 1, 256] paged cache, graph-replayed
    over ``sets`` rotating buffer sets, with a same-size copy beside it.
    ``iters`` > 0 only launches that many times (for ncu captures)."""
    lens = workloads.seeded_uneven_lens(n_tokens, batch, 1)
    last = (torch.tensor(lens).cumsum(0) - 1).to(device)
    cache = workloads.make_cos_sin_cache(16384, 10000.0, device=device)
    blocks = max(1, -(-n_tokens // 64) + 44)
    g = torch.Generator(device=device).manual_seed(0)
    bufs = []
    for _ in range(1 if iters else sets):
        qkv = torch.randn((n_tokens, 8 * 256), generator=g, device=device).to(torch.bfloat16)
        pos = torch.cat([torch.arange(x) for x in lens]).to(device)
        slots = torch.randperm(blocks * 64, generator=g, device=device)[:n_tokens]
        ck = torch.zeros((blocks, 64, 1, 256), dtype=torch.bfloat16, device=device)
        bufs.append((qkv, pos, slots, ck, torch.zeros_like(ck), torch.empty((batch, 6, 256), dtype=torch.bfloat16,
                                                                              device=device), cache.clone()))

    def call(i: int) -> None:
        qkv, pos, slots, ck, cv, q_out, cs = bufs[i % len(bufs)]
        ops.rope_mirror_kv_write(qkv[:, :1536].view(n_tokens, 6, 256), q_out, qkv[:, 1536:1792].view(n_tokens, 1, 256),
                                 qkv[:, 1792:].view(n_tokens, 1, 256), pos, cs, last, slots, ck, cv)

    if iters:
        for i in range(iters):
            call(i)
        torch.cuda.synchronize(device)
        return {"record_type": "launch", "kernel_name": "rope_mirror_kv_write_kernel", "n_tokens": n_tokens,
                "batch_size": batch, "iters": iters}
    for i in range(3):
        call(i)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_launches):
            call(i)
    us = _replay_us(graph, device, trials, replays, graph_launches)
    del graph
    nbytes = kv_write_bytes(n_tokens, batch)
    copy_us = same_size_copy_us(nbytes, sets, device, 5, graph_launches, replays)
    peak, kind = measured_hbm_peak()
    return {
        "record_type": "timing", "case": f"kv_write_n{n_tokens}_bs{batch}", "phase": "prefill_mirror_kv_write",
        "path": "kv_mirror_write", "n_tokens": n_tokens, "batch_size": batch, "us_per_launch": round(us, 3), "bytes_per_launch": nbytes,
        "gb_s": round(nbytes / (us * 1e3), 1), "hbm_frac": round(nbytes / (us * 1e3) / peak, 4),
        "hbm_peak_gbs": peak, "hbm_peak_source": kind, "same_size_copy_us": round(copy_us, 3),
        "frac_of_same_size_copy": round(copy_us / us, 4), "buffer_sets": sets,
        "l2_cold": sets * nbytes > 2 * L2_BYTES, "device_name": torch.cuda.get_device_name(device),
    }


def time_fused_qkv(n_tokens: int, device: torch.device, trials: int = 7, graph_launches: int = 32,
                   replays: int = 20, sets: Optional[int] = None) -> dict:
    """µs per ordinary prefill on a fused QKV projection output [N, 8 x 256]
    (6 Q heads, the K head, the V head per token), two ways, each
    graph-replayed over the same rotating buffer sets:

    * ``strided``: the op on strided Q / K views of the QKV rows (token stride
      2048 elements), with no copy;
    * ``copy_then_rope``: the producer-side pattern this avoids, a contiguous
      copy of Q out of the QKV rows and then the op on that copy (K stays
      strided).

    Positions are 0..N-1 and each set has its own cos/sin cache copy.  The
    record gives both times and what the strided call saves."""
    cache = workloads.make_cos_sin_cache(max(n_tokens, 1), 10000.0, device=device)
    nbytes = 2056 * n_tokens
    if sets is None:
        sets = int(min(16, max(2, -(-2 * L2_BYTES // max(nbytes, 1)))))
    g = torch.Generator(device=device).manual_seed(0)
    bufs = []
    for _ in range(sets):
        qkv = torch.randn((n_tokens, 8 * 256), generator=g, device=device).to(torch.bfloat16)
        bufs.append((qkv, torch.empty((n_tokens, 6, 256), dtype=torch.bfloat16, device=device),
                     torch.arange(n_tokens, dtype=torch.int64, device=device), cache.clone()))

    def views(qkv: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return qkv[:, :1536].view(n_tokens, 6, 256), qkv[:, 1536:1792].view(n_tokens, 1, 256)

    def strided(i: int) -> None:
        qkv, _, pos, cs = bufs[i % sets]
        q, k = views(qkv)
        ops.welmv4_inplace_rope_npu(q, k, pos, cs)

    def copy_then_rope(i: int) -> None:
        qkv, q_buf, pos, cs = bufs[i % sets]
        q, k = views(qkv)
        q_buf.copy_(q)
        ops.welmv4_inplace_rope_npu(q_buf, k, pos, cs)

    out = {}
    for name, call in (("strided", strided), ("copy_then_rope", copy_then_rope)):
        for i in range(3):
            call(i)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(graph_launches):
                call(i)
        out[name] = _replay_us(graph, device, trials, replays, graph_launches)
        del graph
    peak, kind = measured_hbm_peak()
    us = out["strided"]
    return {
        "record_type": "timing", "case": f"fused_qkv_prefill_m{n_tokens}", "phase": "prefill",
        "path": "fused_qkv_strided", "n_tokens": n_tokens, "q_token_stride": 2048, "k_token_stride": 2048,
        "us_per_launch": round(us, 3), "bytes_per_launch": nbytes, "gb_s": round(nbytes / (us * 1e3), 1),
        "hbm_frac": round(nbytes / (us * 1e3) / peak, 4), "hbm_peak_gbs": peak, "hbm_peak_source": kind,
        "copy_then_rope_us": round(out["copy_then_rope"], 3),
        "saved_us": round(out["copy_then_rope"] - us, 3), "buffer_sets": sets,
        "l2_cold": sets * nbytes > 2 * L2_BYTES, "device_name": torch.cuda.get_device_name(device),
    }


# Dense ordinary launches of at most this many tokens run one head per thread
# (kHeadSplitMaxTokens in csrc/rope_host.cuh).
HEAD_SPLIT_MAX_TOKENS = 3328


def kernel_name(case: workloads.Case) -> str:
    """The kernel a case's launch runs, for ``ncu -k`` filters."""
    if case.is_mirror:
        return "rope_mirror_head_kernel"
    if not case.is_segmented:
        return "rope_ordinary_head_kernel" if case.n_tokens <= HEAD_SPLIT_MAX_TOKENS else "rope_ordinary_stream_kernel"
    # segmented: the streaming kernel over tile slots when at least half of
    # the slots can hold a token (stream_slots in csrc/rope_ordinary.cu)
    tiles = len(workloads.tile_starts_for(case.segment_lens)) - 1
    return "rope_ordinary_stream_kernel" if tiles > 0 and 2 * case.n_tokens >= 64 * tiles else "rope_ordinary_kernel"


def launch_case(case: workloads.Case, device: torch.device, iters: int, from_lens: bool = False,
                gather_only: bool = False) -> dict:
    inp = workloads.make_inputs(case, device)
    if from_lens:
        _with_lens(case, inp, device)
    for _ in range(iters):
        if gather_only:
            ceiling_gather(inp.positions, inp.cache)
        else:
            _launch(inp)
    torch.cuda.synchronize(device)
    return {"record_type": "launch", **case_fields(case), "iters": iters,
            "kernel_name": "ceiling_gather_kernel" if gather_only else kernel_name(case)}


def write_csv(records: list[dict], path: str) -> None:
    """Records as one CSV table over the union of their fields, in first-seen
    order (the reference writes its records this way,
    bench_welmv4_inplace_rope_npu.py:2178-2188); nested fields are JSON."""
    import csv

    fields: list[str] = []
    for rec in records:
        fields.extend(k for k in rec if k not in fields)
    with open(path, "w", newline="") as fh:
        writer = csv.DictWriter(fh, fieldnames=fields)
        writer.writeheader()
        for rec in records:
            writer.writerow({k: json.dumps(v) if isinstance(v, (dict, list)) else v for k, v in rec.items()})


def run(cases: Iterable[workloads.Case], device: torch.device, time_it: bool, iters: int,
        out: Optional[str], from_lens: bool = False, copy_ceiling: bool = False,
        host_transport: Optional[str] = None, shared_cache: bool = False, gather_only: bool = False,
        sets: Optional[int] = None, tma_floor: bool = False) -> list[dict]:
    records = []
    sink = open(out, "a") if out else None
    try:
        for case in cases:
            if host_transport is not None:
                rec = time_host_case(case, device, host_transport)
            elif time_it:
                rec = time_case(case, device, from_lens=from_lens, copy_ceiling=copy_ceiling,
                                shared_cache=shared_cache, sets=sets, tma_floor=tma_floor)
            else:
                rec = launch_case(case, device, iters, from_lens, gather_only)
            records.append(rec)
            line = json.dumps(rec)
            print(line, flush=True)
            if sink:
                sink.write(line + "\n")
                sink.flush()
    finally:
        if sink:
            sink.close()
    return records


def main(argv: Optional[list[str]] = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--cases", default="b_prefill_m16384",
                        help="case names or groups (reference, baseline, decode, prefill, mirror, segmented)")
    parser.add_argument("--time", action="store_true", help="time each case (graph replay, rotating buffers)")
    parser.add_argument("--iters", type=int, default=20, help="eager launches per case (without --time)")
    parser.add_argument("--device", default="cuda:0")
    parser.add_argument("--json", default=None, help="append JSON lines here")
    parser.add_argument("--csv", default=None, help="write all records as one CSV table here")
    parser.add_argument("--shared-cache", action="store_true",
                        help="with --time: one cos/sin cache for all buffer sets (hot in L2, as in serving)")
    parser.add_argument("--sets", type=int, default=None,
                        help="with --time: rotate this many buffer sets (the copy ceilings too) instead of "
                             "enough to keep L2 cold; 1 or 2 keep every byte L2-resident")
    parser.add_argument("--tma-floor", action="store_true",
                        help="with --time (dense ordinary cases): also time the TMA-staged slice mover "
                             "(welm_rope_ceiling_tma_slices) on the same buffers")
    parser.add_argument("--mirror-from-lens", action="store_true",
                        help="run segmented KV-mirror cases through rope_mirror_from_lens")
    parser.add_argument("--copy-ceiling", action="store_true",
                        help="with --time: also time a same-size device copy (the practical ceiling)")
    parser.add_argument("--gather-only", action="store_true",
                        help="with --iters: launch only the position and cos/sin gather (welm_rope_ceiling_gather) "
                             "on the case's positions, for profiling it apart from the Q/K slices")
    parser.add_argument("--host", choices=("mapped", "staged"), default=None,
                        help="time the host-memory entry on pinned Q/K with this transport (ordinary cases)")
    parser.add_argument("--kv-write", default=None, metavar="N,BS",
                        help="time the fused KV-mirror cache write for N tokens in BS requests (with --iters: "
                             "only launch it)")
    parser.add_argument("--fused-qkv", type=int, default=None, metavar="M",
                        help="time prefill on strided Q/K views of an [M, 8 x 256] QKV output against a "
                             "contiguous Q copy followed by the op")
    args = parser.parse_args(argv)
    if args.sets is not None and args.sets < 1:
        parser.error("--sets needs at least 1")
    if not torch.cuda.is_available():
        print("the launcher needs a CUDA device", file=sys.stderr)
        return 2
    device = torch.device(args.device)
    torch.cuda.set_device(device)
    if args.kv_write or args.fused_qkv:
        if args.fused_qkv:
            if args.fused_qkv <= 0:
                parser.error("--fused-qkv needs a positive token count")
            rec = time_fused_qkv(args.fused_qkv, device)
        else:
            n, bs = (int(x) for x in args.kv_write.split(","))
            rec = time_kv_write(n, bs, device, iters=0 if args.time else args.iters)
        print(json.dumps(rec), flush=True)
        if args.json:
            with open(args.json, "a") as fh:
                fh.write(json.dumps(rec) + "\n")
        return 0
    records = run(select_cases(args.cases), device, args.time, args.iters, args.json, args.mirror_from_lens,
                  args.copy_ceiling, args.host, args.shared_cache, args.gather_only, args.sets, args.tma_floor)
    if args.csv:
        write_csv(records, args.csv)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
