"""CUDA-graph capture and replay with the producer inside the graph.

Every graph below copies fresh inputs into the op's buffers (the producer)
and then launches the op, so each replay's kernel starts, under programmatic
dependent launch, while its producer may still run.  Between replays the
sources change, so the hints a kernel reads before its dependency wait are
stale on purpose: the results must still equal the oracle for the new
inputs bit for bit.  This is the launch pattern the benchmark times.
"""

from __future__ import annotations

import pytest
import torch

import testfiles_b200 as welm
from oracle import rope_oracle
from testfiles_b200 import workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAXPOS = 4096


def capture(step):
    step()  # first call outside the capture (library load, lazy setup)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    return graph


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().view(torch.int16)


def seeded(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.bfloat16)


def within_request_positions(lens):
    return torch.cat([torch.arange(n, dtype=torch.int64) for n in lens])


@pytest.fixture(scope="module")
def cache():
    host = workloads.make_cos_sin_cache(MAXPOS, 10000.0)
    return host, host.to(DEV)


def test_ordinary_prefill_replays_with_fresh_inputs(cache):
    host_cache, dev_cache = cache
    m = 3000
    src = [torch.empty((m, 6, 256), dtype=torch.bfloat16, device=DEV),
           torch.empty((m, 1, 256), dtype=torch.bfloat16, device=DEV),
           torch.empty(m, dtype=torch.int64, device=DEV)]
    q, k, p = (torch.empty_like(t) for t in src)

    def load(seed):
        g = torch.Generator().manual_seed(seed)
        host = (seeded((m, 6, 256), seed), seeded((m, 1, 256), seed + 1),
                torch.randint(0, MAXPOS, (m,), generator=g, dtype=torch.int64))
        for s, h in zip(src, host):
            s.copy_(h)
        return host

    def step():
        q.copy_(src[0])
        k.copy_(src[1])
        p.copy_(src[2])
        welm.welmv4_inplace_rope_npu(q, k, p, dev_cache)

    load(1)
    graph = capture(step)
    for seed in (11, 12, 13):
        hq, hk, hp = load(seed)
        graph.replay()
        torch.cuda.synchronize()
        q_ref, k_ref = rope_oracle.reference_outputs(hq, hk, hp, None, host_cache)
        assert torch.equal(bits(q), q_ref.view(torch.int16)), seed
        assert torch.equal(bits(k), k_ref.view(torch.int16)), seed


# Same total length and tile count, different request boundaries: the table
# and last_index the device builder writes change from replay to replay.
LENS_SETS = ([100, 200, 300], [300, 200, 100], [150, 150, 300])


@pytest.mark.parametrize("entry", ["builder+table", "from_lens"])
def test_segmented_mirror_replays_with_moving_request_boundaries(cache, entry):
    host_cache, dev_cache = cache
    n, bs = 600, 3
    tiles = {welm.count_segment_tiles(lens) for lens in LENS_SETS}
    assert tiles == {11}
    lens_src = torch.empty(bs, dtype=torch.int64, device=DEV)
    q_src = torch.empty((bs, 6, 256), dtype=torch.bfloat16, device=DEV)
    k_src = torch.empty((n, 1, 256), dtype=torch.bfloat16, device=DEV)
    p_src = torch.empty(n, dtype=torch.int64, device=DEV)
    lens_dev, q, k, p = (torch.empty_like(t) for t in (lens_src, q_src, k_src, p_src))
    capacity = -(-n // 64) + bs + 1

    def load(lens, seed):
        host = (torch.tensor(lens, dtype=torch.int64), seeded((bs, 6, 256), seed), seeded((n, 1, 256), seed + 1),
                within_request_positions(lens))
        for s, h in zip((lens_src, q_src, k_src, p_src), host):
            s.copy_(h)
        return host

    def step():
        lens_dev.copy_(lens_src)
        q.copy_(q_src)
        k.copy_(k_src)
        p.copy_(p_src)
        if entry == "from_lens":
            welm.rope_mirror_from_lens(q, k, p, dev_cache, lens_dev)
        else:
            starts, _, last = welm.build_segment_tile_starts_device(lens_dev, capacity)
            welm.rope_mirror_prefill(q, k, p, dev_cache, last, starts, 11, n, bs, q.stride(0), k.stride(0), 1)

    load(LENS_SETS[0], 1)
    graph = capture(step)
    for i, lens in enumerate(LENS_SETS * 2):
        _, hq, hk, hp = load(lens, 20 + i)
        graph.replay()
        torch.cuda.synchronize()
        last = torch.tensor(rope_oracle.make_last_index(n, bs, lens), dtype=torch.int64)
        q_ref, k_ref = rope_oracle.reference_outputs(hq, hk, hp, last, host_cache)
        assert torch.equal(bits(q), q_ref.view(torch.int16)), lens
        assert torch.equal(bits(k), k_ref.view(torch.int16)), lens


# Ordinary segmented prefill with the device builder in the graph: the table
# changes from replay to replay (same tile count), so tile-slot items whose
# pre-wait table hints name another token must reload.  The lengths sum to
# fewer than N tokens, so the tail stays unrotated.  "slots": most slots
# live (streaming kernel over tile slots); "table": 40 short requests, so
# most slots are empty (token-mapped kernel over the staged table).
ORDINARY_LENS_SETS = {
    "slots": ([100, 200, 250], [250, 200, 100], [150, 150, 250]),
    "table": tuple([(7 * i + s) % 10 + 1 for i in range(40)] for s in (0, 3, 6)),
}


@pytest.mark.parametrize("kind", sorted(ORDINARY_LENS_SETS))
def test_segmented_prefill_replays_with_moving_request_boundaries(cache, kind):
    host_cache, dev_cache = cache
    sets = ORDINARY_LENS_SETS[kind]
    n, bs = 600, len(sets[0])
    tiles = {welm.count_segment_tiles(lens) for lens in sets}
    assert len(tiles) == 1
    tiles = tiles.pop()
    assert all(sum(lens) <= n for lens in sets)
    lens_src = torch.empty(bs, dtype=torch.int64, device=DEV)
    q_src = torch.empty((n, 6, 256), dtype=torch.bfloat16, device=DEV)
    k_src = torch.empty((n, 1, 256), dtype=torch.bfloat16, device=DEV)
    p_src = torch.empty(n, dtype=torch.int64, device=DEV)
    lens_dev, q, k, p = (torch.empty_like(t) for t in (lens_src, q_src, k_src, p_src))
    capacity = -(-n // 64) + bs + 1

    def load(lens, seed):
        pos = within_request_positions(lens)
        pos = torch.cat([pos, torch.zeros(n - pos.numel(), dtype=torch.int64)])
        host = (torch.tensor(lens, dtype=torch.int64), seeded((n, 6, 256), seed), seeded((n, 1, 256), seed + 1), pos)
        for s, h in zip((lens_src, q_src, k_src, p_src), host):
            s.copy_(h)
        return host

    def step():
        lens_dev.copy_(lens_src)
        q.copy_(q_src)
        k.copy_(k_src)
        p.copy_(p_src)
        starts, _, _ = welm.build_segment_tile_starts_device(lens_dev, capacity)
        welm.rope_prefill(q, k, p, dev_cache, starts, tiles, n, q.stride(0), k.stride(0), 1)

    load(sets[0], 1)
    graph = capture(step)
    for i, lens in enumerate(sets * 2):
        _, hq, hk, hp = load(lens, 40 + i)
        graph.replay()
        torch.cuda.synchronize()
        table = rope_oracle.build_tile_starts(lens)
        q_ref, k_ref = rope_oracle.tiled_outputs(hq, hk, hp, host_cache, tiles, 1, table)
        assert torch.equal(bits(q), q_ref.view(torch.int16)), lens
        assert torch.equal(bits(k), k_ref.view(torch.int16)), lens
