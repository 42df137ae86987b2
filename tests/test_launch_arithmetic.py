"""CPU checks of the launch arithmetic of the one-head kernel, the streaming
kernel, the one-head mirror (dense and tile-slot items) and the ceiling copy:
the grid the host computes covers every item exactly once and every index a
thread forms stays inside its buffer.  The rules are restated from
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
HEAD_FEW_CTAS = int(re.search(r"constexpr int64_t kHeadFewCtas = (\d+);", SRC).group(1))


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
    if items <= HEAD_FEW_CTAS * BLOCK:
        grid, block = (items + BLOCK - 1) // BLOCK, BLOCK
    else:
        grid, block = shape_for(items)
    return (grid, block) if grid * block >= items else None


@pytest.mark.parametrize("tokens", [1, 2, 3, 17, 22, 23, 127, 128, 338, 1353, 1354, 2048, 3327, 3328])
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
    # decode batches up to 22 tokens run in at most kHeadFewCtas 128-thread CTAs
    assert head_split_shape(22) == (5, BLOCK) and head_split_shape(23)[1] == 32


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
    assert "shape = items <= kHeadFewCtas * kBlock ? LaunchShape{unsigned((items + kBlock - 1) / kBlock)" in SRC
    assert "const int64_t wave = int64_t(sms > 0 ? sms : 1) * 16 * kBlock;" in ceiling
    assert "const int64_t need = (vectors + 4 * kBlock - 1) / (4 * kBlock);" in ceiling


STREAM_CTAS = int(re.search(r"constexpr int kStreamCtasPerSm = (\d+);", SRC).group(1))
Q_HEADS = 6
TILE = 64


def stream_shape(items: int) -> tuple[int, int]:
    if 64 < items <= 3 * SMS * BLOCK:
        return (items + 31) // 32, 32
    need = (items + BLOCK - 1) // BLOCK
    return min(need, SMS * STREAM_CTAS), BLOCK


def launch_heads(total: int) -> tuple[int, int]:
    if total <= SMS * BLOCK:
        return (total + 31) // 32, 32
    return (total + BLOCK - 1) // BLOCK, BLOCK


@pytest.mark.parametrize("tokens", [3329, 4096, 9472, 9473, 14208, 14209, 16384, 18944, 18945, 40000, 150000])
def test_streaming_grid_stride_covers_every_item_once(tokens):
    """rope_ordinary_stream_kernel: item = first + k * stride for k = 0, 1, ...
    with stride = grid x block; every (token, part) item is visited once."""
    items = tokens * PARTS
    grid, block = stream_shape(items)
    stride = grid * block
    hits = np.zeros(items, dtype=np.int32)
    first = np.arange(stride, dtype=np.int64)
    cur = first[first < items]
    while cur.size:
        np.add.at(hits, cur, 1)
        cur = cur + stride
        cur = cur[cur < items]
    assert hits.min() == 1 and hits.max() == 1
    # up to 18944 tokens every thread owns at most one item (the prefetch
    # before the wait covers all of them); above that the loop prefetches ahead
    assert (items <= stride) == (tokens <= SMS * STREAM_CTAS * BLOCK // PARTS)


@pytest.mark.parametrize("rows,tokens", [(1, 16384), (128, 16384), (3, 1), (2048, 5000), (0, 700)])
def test_mirror_one_head_items_decode_inside_their_buffers(rows, tokens):
    """rope_mirror_head_kernel (dense): Q items (row * 6 + head) * 4 + part,
    then K items token * 4 + part; one item per thread, every item once."""
    q_items, k_items = rows * Q_HEADS * PARTS, tokens * PARTS
    total = q_items + k_items
    grid, block = launch_heads(total)
    item = np.arange(grid * block, dtype=np.int64)
    assert grid * block >= total and (grid - 1) * block < total
    is_q = item < q_items
    is_k = ~is_q & (item - q_items < k_items)
    slc = item >> 2
    row, head = slc // Q_HEADS, slc % Q_HEADS
    tok = (item - q_items) >> 2
    assert (row[is_q] < rows).all() and (head[is_q] < Q_HEADS).all()
    assert (tok[is_k] < tokens).all() and (tok[is_k] >= 0).all()
    assert is_q.sum() == q_items and is_k.sum() == k_items


@pytest.mark.parametrize("tiles", [1, 64, 320, 479, 3600])
def test_tile_slot_items_map_into_the_table(tiles):
    """Slot items (mirror and the streaming segmented path): slot = item / 4,
    tile = slot / 64, j = slot % 64; every slot of every tile once, and the
    table entries a slot reads are tile and tile + 1 <= T."""
    k_items = tiles * TILE * PARTS
    grid, block = launch_heads(k_items)
    s_grid, s_block = stream_shape(k_items)
    if s_block == BLOCK:  # the segmented ordinary launch takes one item per thread
        s_grid = (k_items + BLOCK - 1) // BLOCK
    for g, b in ((grid, block), (s_grid, s_block)):
        item = np.arange(g * b, dtype=np.int64)
        live = item < k_items
        slot = item[live] >> 2
        tile, j = slot // TILE, slot % TILE
        assert tile.max() + 1 <= tiles and j.max() < TILE
        assert np.array_equal(np.sort(item[live]), np.arange(k_items))


def test_restated_stream_and_head_rules_match_the_sources():
    mirror = (REPO / "testfiles_b200" / "csrc" / "rope_mirror.cu").read_text()
    ordinary = (REPO / "testfiles_b200" / "csrc" / "rope_ordinary.cu").read_text()
    assert "if (sms > 0 && items > 64 && items <= 3 * int64_t(sms) * kBlock) return {unsigned((items + 31) / 32), 32u};" in SRC
    assert "const int64_t cap = sms > 0 ? int64_t(sms) * kStreamCtasPerSm : need;" in SRC
    assert "if (sms > 0 && total <= int64_t(sms) * kBlock) return launch(kernel, unsigned((total + 31) / 32), 32u, 0, s, a);" in mirror
    assert "h.q_items = int32_t(rows * kQHeads * kParts);" in mirror
    assert "h.k_items = int32_t(int64_t(a.num_tiles) * kTile * kParts);" in mirror
    assert "if (shape.block == unsigned(kBlock)) shape.grid = unsigned((int64_t(h.k_items) + kBlock - 1) / kBlock);" in ordinary
    assert "bool stream_slots(int64_t num_tiles, int64_t n_tokens) { return num_tiles > 0 && 2 * n_tokens >= num_tiles * kTile; }" in ordinary
