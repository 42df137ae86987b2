"""Seeded random configurations through every entry and launch route,
against the oracle bit for bit.

Each seed draws one configuration: the entry (ordinary dense, ordinary
segmented, KV mirror dense, KV mirror segmented, KV mirror from request
lengths), the sizes (decode batches that take the few-CTA shape, one-head
launches, streaming launches; dense and sparse tile tables), the memory
layout of Q and K (packed, fused QKV views, padded token strides, and
strides or bases that force the scalar path) and the positions (random, or
per-request runs from a random offset as in chunked prefill).  The results
must equal the oracle's exactly, the status word must stay clear, and no
byte outside the Q and K views may change.
"""

from __future__ import annotations

import random

import pytest
import torch

import testfiles_b200 as welm
from oracle import rope_oracle
from testfiles_b200 import workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAX_POSITION = 8192
ENTRIES = ("ordinary", "ordinary_segmented", "mirror", "mirror_segmented", "mirror_from_lens")
LAYOUTS = ("packed", "fused_qkv", "padded", "scalar")


@pytest.fixture(scope="module")
def cache():
    host = workloads.make_cos_sin_cache(MAX_POSITION, 10000.0)
    return host, host.to(DEV)


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().view(torch.int16)


class Rows:
    """A [rows, heads, 256] bf16 view inside a larger device buffer whose other
    bytes are filled with a sentinel, so writes outside the view show up."""

    def __init__(self, data: torch.Tensor, token_stride: int, offset: int, head_offset: int = 0):
        rows, heads, lanes = data.shape
        size = offset + head_offset + (rows - 1) * token_stride + heads * lanes + 16 if rows else 16
        self.store = torch.full((size,), -7.0, dtype=torch.bfloat16, device=DEV)
        self.view = self.store.as_strided(data.shape, (token_stride, lanes, 1), offset + head_offset)
        if rows:
            self.view.copy_(data.to(DEV))
        self.before = self.store.clone()
        self.mask = torch.ones_like(self.store, dtype=torch.bool)
        if rows:
            self.mask.as_strided(data.shape, (token_stride, lanes, 1), offset + head_offset).fill_(False)

    def outside_unchanged(self) -> bool:
        return torch.equal(self.store[self.mask], self.before[self.mask])


def place(q: torch.Tensor, k: torch.Tensor, layout: str, rng: random.Random) -> tuple[Rows, Rows]:
    if layout == "packed":
        return Rows(q, 6 * 256, 0), Rows(k, 256, 0)
    if layout == "fused_qkv":  # Q heads 0..5 and K head 6 of an [rows, 8 x 256] projection output
        return Rows(q, 8 * 256, 0), Rows(k, 8 * 256, 0, head_offset=6 * 256)
    if layout == "padded":  # token strides that keep 16-byte vectors
        return Rows(q, 6 * 256 + 8 * rng.randint(1, 8), 0), Rows(k, 256 + 8 * rng.randint(1, 8), 0)
    # scalar path: a token stride that is not a multiple of 8 elements, or a base off 16 bytes
    if rng.random() < 0.5:
        return Rows(q, 6 * 256 + rng.choice((1, 3, 5)), 0), Rows(k, 256 + rng.choice((1, 2, 7)), 0)
    return Rows(q, 6 * 256, rng.choice((1, 2, 3))), Rows(k, 256, rng.choice((1, 5)))


def draw_lens(rng: random.Random, sparse: bool) -> list[int]:
    bs = rng.randint(1, 48)
    if sparse:  # short requests: most of each request's 64-token tile is empty
        return [rng.randint(1, 12) for _ in range(bs)]
    return [rng.choice((64, 128, rng.randint(1, 400))) for _ in range(bs)]


def request_positions(lens: list[int], rng: random.Random) -> torch.Tensor:
    runs = []
    for n in lens:
        start = rng.randint(0, MAX_POSITION - n) if rng.random() < 0.5 else 0
        runs.append(torch.arange(start, start + n, dtype=torch.int64))
    return torch.cat(runs) if runs else torch.zeros(0, dtype=torch.int64)


def draw_ordinary_tokens(rng: random.Random) -> int:
    band = rng.random()
    if band < 0.3:
        return rng.randint(1, 22)  # few 128-thread CTAs
    if band < 0.7:
        return rng.randint(23, 3328)  # one head per thread
    return rng.randint(3329, 12000)  # streaming kernel


@pytest.mark.parametrize("seed", range(240))
def test_random_configuration_matches_oracle(cache, seed):
    host_cache, dev_cache = cache
    rng = random.Random(1000 + seed)
    entry = ENTRIES[seed % len(ENTRIES)]
    layout = LAYOUTS[(seed // len(ENTRIES)) % len(LAYOUTS)]
    g = torch.Generator().manual_seed(seed)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)

    if entry == "ordinary":
        n = draw_ordinary_tokens(rng)
        pos = torch.randint(0, MAX_POSITION, (n,), generator=g, dtype=torch.int64)
        lens, table, last, rows = None, None, None, n
    else:
        lens = draw_lens(rng, sparse=entry == "ordinary_segmented" and rng.random() < 0.4)
        n = sum(lens)
        pos = request_positions(lens, rng)
        table = rope_oracle.build_tile_starts(lens)
        last = torch.tensor(rope_oracle.make_last_index(n, len(lens), lens), dtype=torch.int64)
        rows = n if entry == "ordinary_segmented" else len(lens)
        if entry == "mirror":  # dense mirror: every token, Q rows at arbitrary tokens
            last = torch.randint(0, n, (len(lens),), generator=g, dtype=torch.int64)

    q = torch.randn((rows, 6, 256), generator=g).to(torch.bfloat16)
    k = torch.randn((n, 1, 256), generator=g).to(torch.bfloat16)
    qd, kd = place(q, k, layout, rng)
    pd = pos.to(DEV)

    if entry == "ordinary":
        welm.welmv4_inplace_rope_npu(qd.view, kd.view, pd, dev_cache, status=status)
        q_ref, k_ref = rope_oracle.reference_outputs(q, k, pos, None, host_cache)
    elif entry == "ordinary_segmented":
        starts = torch.tensor(table, dtype=torch.int32, device=DEV)
        welm.welmv4_inplace_rope_npu(qd.view, kd.view, pd, dev_cache, None, starts, status=status)
        q_ref, k_ref = rope_oracle.tiled_outputs(q, k, pos, host_cache, len(table) - 1, 1, table)
    elif entry == "mirror":
        welm.welmv4_inplace_rope_npu(qd.view, kd.view, pd, dev_cache, last.to(DEV), status=status)
        q_ref, k_ref = rope_oracle.tiled_outputs(q, k, pos, host_cache, -(-n // 64), 0, None, last)
    elif entry == "mirror_segmented":
        starts = torch.tensor(table, dtype=torch.int32, device=DEV)
        welm.welmv4_inplace_rope_npu(qd.view, kd.view, pd, dev_cache, last.to(DEV), starts, status=status)
        q_ref, k_ref = rope_oracle.tiled_outputs(q, k, pos, host_cache, len(table) - 1, 1, table, last)
    else:
        lens_dev = torch.tensor(lens, dtype=torch.int64, device=DEV)
        welm.rope_mirror_from_lens(qd.view, kd.view, pd, dev_cache, lens_dev, status=status)
        q_ref, k_ref = rope_oracle.tiled_outputs(q, k, pos, host_cache, len(table) - 1, 1, table, last)
    torch.cuda.synchronize()

    what = f"seed {seed}: {entry}, {layout}, N={n}, rows={rows}"
    assert torch.equal(bits(qd.view), q_ref.view(torch.int16)), what + " (query)"
    assert torch.equal(bits(kd.view), k_ref.view(torch.int16)), what + " (key)"
    assert status.item() == 0, what
    assert qd.outside_unchanged() and kd.outside_unchanged(), what + " (bytes outside the views)"
