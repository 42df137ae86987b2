"""CPU checks of the launch arithmetic of the one-head kernel and the ceiling
copy: the grid the host computes covers every item exactly once and every
index a thread forms stays inside its buffer.  The rules are restated from
testfiles_b200/csrc/rope_host.cuh and rope_ceiling.cu for a B200's 148 SMs;
the constants are read from the header so the two cannot drift apart."""

from __future__ import annotations

import re

import numpy as np
import pytest

from conftest import REPO

SMS = 148
BLOCK = 128
PARTS = 4
HEADS = 7  # the K head and six Q heads
SRC = (REPO / "testfiles_b200" / "csrc" / "rope_host.cuh").read_text()
HEAD_SPLIT_MAX = int(re.search(r"constexpr int64_t kHeadSplitMaxTokens = (\d+);", SRC).group(1))


def grid_for(items: int) -> int:
    need = (items + BLOCK - 1) // BLOCK
    return min(need, SMS * 16)


def shape_for(total: int) -> tuple[int, int]:
    if 2 * 32 < total <= 2 * SMS * BLOCK:
        return (total + 31) // 32, 32
    return grid_for(total), BLOCK


def head_split_shape(tokens: int):
    if tokens > HEAD_SPLIT_MAX:
        return None
    items = tokens * HEADS * PARTS
    grid, block = shape_for(items)
    return (grid, block) if grid * block >= items else None


@pytest.mark.parametrize("tokens", [1, 2, 3, 17, 127, 128, 338, 1353, 1354, 2048, 4095, 4096])
def test_one_head_items_cover_every_slice_once(tokens):
    grid, block = head_split_shape(tokens)
    item = np.arange(grid * block)
    live = item < tokens * HEADS * PARTS
    part, slc = item & (PARTS - 1), item >> 2
    tok, head = slc // HEADS, slc % HEADS
    assert live.sum() == tokens * HEADS * PARTS
    assert tok[live].max() < tokens and head[live].max() < HEADS
    keys = (tok[live] * HEADS + head[live]) * PARTS + part[live]
    assert np.array_equal(np.sort(keys), np.arange(tokens * HEADS * PARTS))
    # lanes: 192 + 8 * part + (0..7) for x1 and +32 for x2 stay inside the head
    assert 192 + 8 * (PARTS - 1) + 7 + 32 < 256


def test_one_head_rule_applies_up_to_the_limit_only():
    assert all(head_split_shape(t) is not None for t in range(1, HEAD_SPLIT_MAX + 1))
    assert head_split_shape(HEAD_SPLIT_MAX + 1) is None


@pytest.mark.parametrize("vectors", [1, 127, 303104, 303105, 524288, 1212416, 1310723, 2_100_000])
def test_ceiling_copy_rounds_cover_every_vector_once(vectors):
    wave = SMS * 16 * BLOCK
    if vectors <= wave:
        per, grid = 1, (vectors + BLOCK - 1) // BLOCK
    else:
        per, grid = 4, min((vectors + 4 * BLOCK - 1) // (4 * BLOCK), wave // BLOCK)
    threads = grid * BLOCK
    hits = np.zeros(vectors, dtype=np.int32)
    base = np.arange(threads, dtype=np.int64)
    while base.size:
        for j in range(per):
            idx = base + j * threads
            np.add.at(hits, idx[idx < vectors], 1)
        base = base + threads * per
        base = base[base < vectors]
    assert hits.min() == 1 and hits.max() == 1


def test_table_path_warp_sized_ctas_cover_every_item():
    for total in (1, 31, 33, 16384 + 129, SMS * BLOCK):
        grid = (total + 31) // 32
        assert grid * 32 >= total and (grid - 1) * 32 < total


def test_restated_rules_match_the_sources():
    ceiling = (REPO / "testfiles_b200" / "csrc" / "rope_ceiling.cu").read_text()
    assert "total > 2 * kSmallBlock && total <= 2 * int64_t(sms) * kBlock" in SRC  # shape_for
    assert "const int64_t cap = sms > 0 ? int64_t(sms) * 16 : need;" in SRC  # grid_for
    assert "if (sms > 0 && total <= int64_t(sms) * kBlock)" in SRC  # warp-sized table CTAs
    assert "const int64_t items = tokens * kHeadsPerToken * kParts;" in SRC  # head_split_shape
    assert "const int64_t wave = int64_t(sms > 0 ? sms : 1) * 16 * kBlock;" in ceiling
    assert "const int64_t need = (vectors + 4 * kBlock - 1) / (4 * kBlock);" in ceiling
