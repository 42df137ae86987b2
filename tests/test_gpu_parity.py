"""GPU parity: the sm_100a library against the oracle, bit for bit.

Every case of the reference catalogue (193) and every benchmark configuration
runs through the drop-in entry ``welmv4_inplace_rope_npu`` and through the
reference-shaped launch surfaces (``rope_prefill`` / ``rope_mirror_prefill``
with the reference kernels' integer arguments).  Outputs must equal the
oracle's exactly: lanes 0..191 untouched, lanes 192..255 identical BF16 bits
(the tolerance is zero ulp, stricter than the 1-ulp bar), and equal to the
reference's own output digests from tests/golden where this host's cos/sin
cache matches the fixture host's.
"""

from __future__ import annotations

import random

import pytest
import torch

from conftest import digest
from oracle import rope_oracle
import testfiles_b200 as welm
from testfiles_b200 import _native, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
ALL = workloads.reference_cases() + workloads.baseline_cases()
CASES = {c.name: c for c in ALL}


def mismatch_report(got: torch.Tensor, want: torch.Tensor) -> str:
    g, w = got.float(), want.float()
    diff = (g - w).abs()
    ulp = (got.view(torch.int16).int() - want.view(torch.int16).int()).abs()
    return (f"max_abs_diff={diff.max().item():.3g} mismatches={(ulp != 0).sum().item()} "
            f"max_ulp={ulp.max().item()} prefix_equal={torch.equal(got[..., :192], want[..., :192])}")


def assert_bitexact(got: torch.Tensor, want: torch.Tensor, what: str) -> None:
    got = got.cpu()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"{what}: {mismatch_report(got, want)}"


def run_drop_in(inp: workloads.Inputs, status: torch.Tensor | None = None) -> workloads.Inputs:
    dev = inp.to(DEV)
    welm.welmv4_inplace_rope_npu(dev.query, dev.key, dev.positions, dev.cache, dev.last_index,
                                 dev.segment_tile_starts, status=status)
    torch.cuda.synchronize()
    return dev


@pytest.mark.parametrize("name", sorted(CASES))
def test_drop_in_matches_oracle(name, golden_outputs):
    case = CASES[name]
    inp = workloads.make_inputs(case, "cpu")
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = run_drop_in(inp, status)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert_bitexact(dev.query, q_ref, f"{name} query")
    assert_bitexact(dev.key, k_ref, f"{name} key")
    assert status.item() == 0
    rec = golden_outputs[name]
    if digest(inp.cache) == rec["cache"] and digest(inp.query) == rec["inputs"]["query"]:
        assert digest(dev.query) == rec["outputs"]["query"]
        assert digest(dev.key) == rec["outputs"]["key"]


@pytest.mark.parametrize("name", sorted(c.name for c in workloads.reference_cases()))
def test_reference_launch_surface(name):
    """The reference kernels' argument lists (bench_welmv4_inplace_rope_npu.py:1164-1388)."""
    case = CASES[name]
    inp = workloads.make_inputs(case, "cpu")
    dev = inp.to(DEV)
    placeholder = welm.segment_placeholder(DEV)
    n = case.n_tokens
    starts = dev.segment_tile_starts if case.is_segmented else placeholder
    if case.is_mirror:
        welm.rope_mirror_prefill(dev.query, dev.key, dev.positions, dev.cache, dev.last_index, starts,
                                 dev.num_work_tiles, n, case.batch_size, dev.query.stride(0), dev.key.stride(0),
                                 dev.has_segments)
    else:
        welm.rope_prefill(dev.query, dev.key, dev.positions, dev.cache, starts, dev.num_work_tiles, n,
                          dev.query.stride(0), dev.key.stride(0), dev.has_segments)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert_bitexact(dev.query, q_ref, f"{name} query")
    assert_bitexact(dev.key, k_ref, f"{name} key")


def small_inputs(m: int, seed: int = 0, max_position: int = 4096) -> workloads.Inputs:
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((m, 6, 256), dtype=torch.bfloat16, generator=g)
    k = torch.randn((m, 1, 256), dtype=torch.bfloat16, generator=g)
    pos = torch.randint(0, max_position, (m,), generator=g, dtype=torch.int64)
    cache = workloads.make_cos_sin_cache(max_position, 10000.0)
    return workloads.Inputs(q, k, pos, cache, num_work_tiles=(m + 63) // 64)


@pytest.mark.parametrize("q_pad,k_pad,offset", [(2, 0, 0), (0, 3, 0), (0, 0, 1), (8, 8, 0)])
def test_strided_and_misaligned_views(q_pad, k_pad, offset):
    """Strides that are not multiples of 8 elements or bases off 16 bytes take
    the scalar path; both paths must give the oracle's bits."""
    m = 333
    inp = small_inputs(m, 1)
    q_store = torch.zeros(m * (1536 + q_pad) + offset + 8, dtype=torch.bfloat16, device=DEV)
    k_store = torch.zeros(m * (256 + k_pad) + offset + 8, dtype=torch.bfloat16, device=DEV)
    q = q_store.as_strided((m, 6, 256), (1536 + q_pad, 256, 1), offset)
    k = k_store.as_strided((m, 1, 256), (256 + k_pad, 256, 1), offset)
    q.copy_(inp.query.to(DEV))
    k.copy_(inp.key.to(DEV))
    before_q, before_k = q_store.clone(), k_store.clone()
    welm.welmv4_inplace_rope_npu(q, k, inp.positions.to(DEV), inp.cache.to(DEV))
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert_bitexact(q, q_ref, "query")
    assert_bitexact(k, k_ref, "key")
    # bytes outside the views (padding) are untouched
    mask_q = torch.ones_like(q_store, dtype=torch.bool)
    mask_q.as_strided((m, 6, 256), (1536 + q_pad, 256, 1), offset).fill_(False)
    assert torch.equal(q_store[mask_q], before_q[mask_q])
    mask_k = torch.ones_like(k_store, dtype=torch.bool)
    mask_k.as_strided((m, 1, 256), (256 + k_pad, 256, 1), offset).fill_(False)
    assert torch.equal(k_store[mask_k], before_k[mask_k])


def test_fused_qkv_layout():
    """Q and K as strided views of a packed QKV projection output [M, 8*256]
    (6 Q heads, 1 K head, 1 V head): no contiguous() copy is needed."""
    m = 1000
    inp = small_inputs(m, 2)
    qkv = torch.randn((m, 8 * 256), dtype=torch.bfloat16, device=DEV)
    q = qkv[:, : 6 * 256].view(m, 6, 256)
    k = qkv[:, 6 * 256: 7 * 256].view(m, 1, 256)
    q.copy_(inp.query.to(DEV))
    k.copy_(inp.key.to(DEV))
    v_before = qkv[:, 7 * 256:].clone()
    welm.welmv4_inplace_rope_npu(q, k, inp.positions.to(DEV), inp.cache.to(DEV))
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert_bitexact(q, q_ref, "query")
    assert_bitexact(k, k_ref, "key")
    assert torch.equal(qkv[:, 7 * 256:], v_before)


def test_out_of_range_positions_are_skipped_and_flagged():
    m = 200
    inp = small_inputs(m, 3, max_position=512)
    bad = torch.tensor([0, 17, 64, 199])
    inp.positions[bad] = torch.tensor([512, -1, 1 << 40, -(1 << 40)])
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = run_drop_in(inp, status)
    assert status.item() == _native.DEV_BAD_POSITION
    good = torch.ones(m, dtype=torch.bool)
    good[bad] = False
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query[good], inp.key[good], inp.positions[good], None,
                                                 inp.cache)
    assert_bitexact(dev.query.cpu()[good], q_ref, "query")
    assert_bitexact(dev.key.cpu()[good], k_ref, "key")
    assert torch.equal(dev.query.cpu()[bad], inp.query[bad])
    assert torch.equal(dev.key.cpu()[bad], inp.key[bad])


def test_mirror_bad_last_index_is_skipped_and_flagged():
    n, bs = 300, 5
    inp = small_inputs(n, 4)
    q = torch.randn((bs, 6, 256), dtype=torch.bfloat16)
    last = torch.tensor([10, 299, 300, -1, 150], dtype=torch.int64)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    qd, kd = q.to(DEV), inp.key.to(DEV)
    welm.welmv4_inplace_rope_npu(qd, kd, inp.positions.to(DEV), inp.cache.to(DEV), last.to(DEV), status=status)
    torch.cuda.synchronize()
    assert status.item() == _native.DEV_BAD_LAST_INDEX
    ok = torch.tensor([0, 1, 4])
    q_ref = rope_oracle.apply_reference(q[ok], inp.positions[last[ok]], inp.cache)
    assert_bitexact(qd.cpu()[ok], q_ref, "query")
    assert torch.equal(qd.cpu()[2:4], q[2:4])
    assert_bitexact(kd, rope_oracle.apply_reference(inp.key, inp.positions, inp.cache), "key")


@pytest.mark.parametrize("pad", [0, 2100])
@pytest.mark.parametrize("mirror", [False, True])
def test_irregular_tile_tables_follow_reference_masking(mirror, pad):
    """Tiles longer than 64 rotate only their first 64 tokens; empty tiles and
    tiles past N rotate nothing; non-contiguous positions inside a tile use
    each token's own position (per-token gather).  pad=2100 prepends 1-token
    tiles so the table exceeds the shared-memory path (slot path)."""
    n = 400 + pad
    inp = small_inputs(n, 5)
    table = list(range(pad)) + [pad + x for x in (0, 100, 100, 130, 250, 390, 400)]
    starts = torch.tensor(table, dtype=torch.int32)
    tiles = len(table) - 1
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = inp.to(DEV)
    if mirror:
        last = torch.tensor([99 + pad, 399 + pad], dtype=torch.int64)
        q = torch.randn((2, 6, 256), dtype=torch.bfloat16)
        qd = q.to(DEV)
        welm.rope_mirror_prefill(qd, dev.key, dev.positions, dev.cache, last.to(DEV), starts.to(DEV), tiles, n,
                                 2, 1536, 256, 1, status=status)
        torch.cuda.synchronize()
        q_ref, k_ref = rope_oracle.tiled_outputs(q, inp.key, inp.positions, inp.cache, tiles, 1, table, last)
        assert_bitexact(qd, q_ref, "query")
    else:
        welm.rope_prefill(dev.query, dev.key, dev.positions, dev.cache, starts.to(DEV), tiles, n, 1536, 256, 1,
                          status=status)
        torch.cuda.synchronize()
        q_ref, k_ref = rope_oracle.tiled_outputs(inp.query, inp.key, inp.positions, inp.cache, tiles, 1, table)
        assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")
    assert status.item() == _native.DEV_BAD_TILE


def test_tiles_out_of_bounds_are_skipped():
    n = 128
    inp = small_inputs(n, 6)
    table = torch.tensor([64, 128, 190], dtype=torch.int32)  # second tile lies past N
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = inp.to(DEV)
    welm.rope_prefill(dev.query, dev.key, dev.positions, dev.cache, table.to(DEV), 2, n, 1536, 256, 1,
                      status=status)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.tiled_outputs(inp.query, inp.key, inp.positions, inp.cache, 1, 1, [64, 128])
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")
    assert status.item() == _native.DEV_BAD_TILE


@pytest.mark.parametrize("tiles", [0, 1, 3])
def test_fewer_work_tiles_than_tokens(tiles):
    """has_segments=0 rotates tokens [0, min(N, 64 * num_work_tiles))."""
    n = 300
    inp = small_inputs(n, 7)
    dev = inp.to(DEV)
    welm.rope_prefill(dev.query, dev.key, dev.positions, dev.cache, None, tiles, n, 1536, 256, 0)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.tiled_outputs(inp.query, inp.key, inp.positions, inp.cache, tiles, 0)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")


def test_empty_inputs_are_noops():
    cache = workloads.make_cos_sin_cache(16, 10000.0, device=DEV)
    q = torch.empty((0, 6, 256), dtype=torch.bfloat16, device=DEV)
    k = torch.empty((0, 1, 256), dtype=torch.bfloat16, device=DEV)
    pos = torch.empty(0, dtype=torch.int64, device=DEV)
    welm.welmv4_inplace_rope_npu(q, k, pos, cache)
    welm.welmv4_inplace_rope_npu(q, k, pos, cache, torch.empty(0, dtype=torch.int64, device=DEV))
    torch.cuda.synchronize()
    # KV mirror with no Q rows: K is still rotated
    inp = small_inputs(70, 15)
    dev = inp.to(DEV)
    welm.welmv4_inplace_rope_npu(q, dev.key, dev.positions, dev.cache, torch.empty(0, dtype=torch.int64, device=DEV))
    torch.cuda.synchronize()
    assert_bitexact(dev.key, rope_oracle.apply_reference(inp.key, inp.positions, inp.cache), "key")


def test_nan_and_inf_inputs():
    m = 64
    inp = small_inputs(m, 8)
    inp.query[3, 2, 200] = float("nan")
    inp.query[5, 0, 230] = float("inf")
    inp.key[7, 0, 193] = float("-inf")
    inp.key[9, 0, 10] = float("nan")  # a non-rope lane: copied bit for bit
    dev = run_drop_in(inp)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    for got, want, what in ((dev.query.cpu(), q_ref, "query"), (dev.key.cpu(), k_ref, "key")):
        g, w = got.float(), want.float()
        assert torch.equal(torch.isnan(g), torch.isnan(w)), what
        finite = ~torch.isnan(w)
        assert torch.equal(g[finite], w[finite]), what
        assert torch.equal(got[..., :192].view(torch.int16), want[..., :192].view(torch.int16)), what


def test_position_zero_is_identity_on_device():
    m = 256
    inp = small_inputs(m, 9)
    inp.positions.zero_()
    dev = run_drop_in(inp)
    assert torch.equal(dev.query.cpu(), inp.query)
    assert torch.equal(dev.key.cpu(), inp.key)


def test_grid_stride_beyond_one_wave():
    """More work items than resident threads: the grid-stride loop covers them."""
    m = 150_000
    inp = small_inputs(m, 10, max_position=16384)
    dev = run_drop_in(inp)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")


def test_side_stream_launch():
    inp = small_inputs(777, 11)
    dev = inp.to(DEV)
    stream = torch.cuda.Stream(DEV)
    stream.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(stream):
        welm.welmv4_inplace_rope_npu(dev.query, dev.key, dev.positions, dev.cache)
    stream.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")


def test_custom_op_registration():
    inp = small_inputs(100, 12)
    dev = inp.to(DEV)
    torch.ops.welm_b200.inplace_rope(dev.query, dev.key, dev.positions, dev.cache)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")


def test_python_api_rejects_misuse():
    inp = small_inputs(8, 13).to(DEV)
    with pytest.raises(TypeError):
        welm.welmv4_inplace_rope_npu(inp.query.float(), inp.key, inp.positions, inp.cache)
    with pytest.raises(TypeError):
        welm.welmv4_inplace_rope_npu(inp.query, inp.key, inp.positions.int(), inp.cache)
    with pytest.raises(ValueError):
        welm.welmv4_inplace_rope_npu(inp.query[:4], inp.key, inp.positions, inp.cache)
    with pytest.raises(ValueError):
        welm.rope_prefill(inp.query, inp.key, inp.positions, inp.cache, None, 1, 8, 1536, 256, 2)
    with pytest.raises(ValueError):
        welm.welmv4_inplace_rope_npu(inp.query.cpu(), inp.key, inp.positions, inp.cache)


# ---------------------------------------------------------------------------
# Device tile builder.
# ---------------------------------------------------------------------------
def device_build(lens: list[int], capacity: int | None = None):
    t = torch.tensor(lens, dtype=torch.int64, device=DEV)
    total = sum(max(x, 0) for x in lens)
    cap = capacity if capacity is not None else (total + 63) // 64 + len(lens) + 1
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    starts, num_tiles, last = welm.build_segment_tile_starts_device(t, cap, status)
    torch.cuda.synchronize()
    return starts.cpu(), int(num_tiles.item()), last.cpu(), int(status.item())


def test_device_builder_matches_reference_tables(tile_tables):
    for name, rec in tile_tables.items():
        starts, tiles, last, status = device_build(rec["segment_lens"])
        assert status == 0
        assert starts[: tiles + 1].tolist() == rec["segment_tile_starts"], name
        if rec["last_index"] is not None:
            assert last.tolist() == rec["last_index"], name


def test_device_builder_random_lengths_match_host_twin():
    rng = random.Random(3)
    for bs in (0, 1, 2, 31, 32, 1023, 1024, 1025, 3000, 5000):
        lens = [rng.choice([0, 1, 63, 64, 65, 128, rng.randint(0, 2000)]) for _ in range(bs)]
        starts, tiles, last, status = device_build(lens)
        h_starts, h_tiles, h_last = welm.build_segment_tile_starts(lens)
        assert status == 0
        assert tiles == h_tiles
        assert starts[: tiles + 1].tolist() == h_starts.tolist()
        assert last.tolist() == h_last.tolist()


def test_device_builder_flags_overflow_and_negative_lengths():
    _, tiles, _, status = device_build([100, 100], capacity=3)  # needs 5 slots
    assert tiles == 4 and status & _native.DEV_BAD_TILE
    starts, tiles, _, status = device_build([64, -5, 64])
    assert status == _native.DEV_BAD_LENGTH
    assert starts[: tiles + 1].tolist() == [0, 64, 128]


def test_device_built_tables_drive_the_mirror_kernel():
    lens = workloads.seeded_uneven_lens(5000, 37, 1)
    case = workloads.Case("adhoc", "prefill_mirror_segmented", 5000, 37, lens, flavour="baseline")
    inp = workloads.make_inputs(case, "cpu")
    dev = inp.to(DEV)
    starts, num_tiles, last = welm.build_segment_tile_starts_device(
        torch.tensor(lens, dtype=torch.int64, device=DEV), (5000 + 63) // 64 + 37 + 1)
    tiles = int(num_tiles.item())
    welm.rope_mirror_prefill(dev.query, dev.key, dev.positions, dev.cache, last, starts, tiles, 5000, 37,
                             1536, 256, 1)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")


@pytest.mark.parametrize("lens", [
    (1,) * 128 + (3968,),            # 190 tiles for 4096 tokens: staged-table kernel (under half the slots live)
    (64,) * 64,                      # every slot live: streaming kernel over tile slots
    tuple(workloads.seeded_uneven_lens(20000, 300, 3)),  # about 80 % of slots live, more than one wave of slots
    (5, 70, 1, 130, 64, 63, 65) * 9,  # partial tiles of every length, just over half the slots live
])
def test_segmented_prefill_routes_match_oracle(lens):
    """Segmented ordinary prefill takes the streaming kernel over tile slots
    when at least half of the slots can hold a token, else the kernel over the
    staged table; both must equal the oracle."""
    n = sum(lens)
    case = workloads.Case("adhoc_routes", "segmented_prefill", n, 0, lens, flavour="baseline")
    inp = workloads.make_inputs(case, "cpu")
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = run_drop_in(inp, status)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")
    assert status.item() == 0


@pytest.mark.parametrize("mirror", [False, True])
def test_large_tile_tables_match_oracle(mirror):
    """Thousands of short requests: more tiles than the shared-memory table
    holds, so the slot mapping runs; results must still equal the oracle."""
    lens = workloads.seeded_uneven_lens(40000, 3000, 9)
    phase = "prefill_mirror_segmented" if mirror else "segmented_prefill"
    case = workloads.Case("adhoc_large_table", phase, 40000, 3000 if mirror else 0, lens, flavour="baseline")
    inp = workloads.make_inputs(case, "cpu")
    assert inp.num_work_tiles + 1 > 2048
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = run_drop_in(inp, status)
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert_bitexact(dev.query, q_ref, "query")
    assert_bitexact(dev.key, k_ref, "key")
    assert status.item() == 0


@pytest.mark.parametrize("pad", [0, 2100])
def test_non_monotone_tables_are_flagged_and_stay_in_bounds(pad):
    """A table that runs backwards is outside the reference's contract: the
    call must flag it and leave lanes 0..191 alone (every access stays inside
    the K/Q rows by construction)."""
    n = 300 + pad
    inp = small_inputs(n, 14)
    table = list(range(pad)) + [pad + x for x in (0, 64, 32, 96, 300)]
    starts = torch.tensor(table, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dev = inp.to(DEV)
    welm.rope_prefill(dev.query, dev.key, dev.positions, dev.cache, starts, len(table) - 1, n, 1536, 256, 1,
                      status=status)
    torch.cuda.synchronize()
    assert status.item() & _native.DEV_BAD_TILE
    assert torch.equal(dev.query.cpu()[..., :192], inp.query[..., :192])
    assert torch.equal(dev.key.cpu()[..., :192], inp.key[..., :192])


# ---------------------------------------------------------------------------
# KV mirror straight from request lengths (no tile table, no last_index).
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("lens", [
    [16384], [4096, 4096], list(workloads.seeded_uneven_lens(16384, 128, 4)), [1] * 2048,
    [0, 5, 0, 64, 65, 1, 0, 300], list(workloads.reference_uneven_lens(9616, 8)),
])
def test_mirror_from_lens_matches_oracle(lens):
    n = sum(lens)
    case = workloads.Case("adhoc_lens", "prefill_mirror_segmented", n, len(lens), tuple(lens), flavour="baseline")
    inp = workloads.make_inputs(case, "cpu")
    dev = inp.to(DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    welm.rope_mirror_from_lens(dev.query, dev.key, dev.positions, dev.cache,
                               torch.tensor(lens, dtype=torch.int64, device=DEV), status=status)
    torch.cuda.synchronize()
    ends = torch.tensor(lens).cumsum(0)
    valid_q = ends > 0  # a leading zero-length request has no last token
    q_ref = rope_oracle.apply_reference(inp.query[valid_q], inp.positions[ends[valid_q] - 1], inp.cache)
    k_ref = rope_oracle.apply_reference(inp.key, inp.positions, inp.cache)
    assert_bitexact(dev.query.cpu()[valid_q], q_ref, "query")
    assert torch.equal(dev.query.cpu()[~valid_q], inp.query[~valid_q])
    assert_bitexact(dev.key, k_ref, "key")
    assert status.item() == (0 if bool(valid_q.all()) else _native.DEV_BAD_LAST_INDEX)


def test_mirror_from_lens_partial_and_negative_lengths():
    n = 500
    inp = small_inputs(n, 16)
    q = torch.randn((3, 6, 256), dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lens = torch.tensor([100, -7, 250], dtype=torch.int64)  # sum (negative as 0) = 350 < N
    dev = inp.to(DEV)
    qd = q.to(DEV)
    welm.rope_mirror_from_lens(qd, dev.key, dev.positions, dev.cache, lens.to(DEV), status=status)
    torch.cuda.synchronize()
    assert status.item() == _native.DEV_BAD_LENGTH
    k_got = dev.key.cpu()
    assert_bitexact(k_got[:350], rope_oracle.apply_reference(inp.key[:350], inp.positions[:350], inp.cache), "key")
    assert torch.equal(k_got[350:], inp.key[350:])
    last = torch.tensor([99, 99, 349])
    assert_bitexact(qd, rope_oracle.apply_reference(q, inp.positions[last], inp.cache), "query")


def test_launches_without_programmatic_dependent_launch():
    """WELM_ROPE_PDL=0 launches plainly (no early scheduling); results are the
    same bits.  The switch is read once per process, so a child runs it."""
    import subprocess
    import sys
    import textwrap

    from conftest import REPO

    code = textwrap.dedent("""
        import torch, testfiles_b200 as welm
        from oracle import rope_oracle
        from testfiles_b200 import workloads
        for name in ("b_prefill_m577", "b_mirror_segmented_n8192_bs16_uneven", "b_decode_m3"):
            inp = workloads.make_inputs(workloads.find_case(name), "cpu")
            d = inp.to("cuda:0")
            welm.welmv4_inplace_rope_npu(d.query, d.key, d.positions, d.cache, d.last_index, d.segment_tile_starts)
            torch.cuda.synchronize()
            q, k = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
            assert torch.equal(d.query.cpu().view(torch.int16), q.view(torch.int16)), name
            assert torch.equal(d.key.cpu().view(torch.int16), k.view(torch.int16)), name
        print("ok")
    """)
    env = dict(__import__("os").environ, WELM_ROPE_PDL="0")
    out = subprocess.run([sys.executable, "-c", code], cwd=REPO, env=env, capture_output=True, text=True, timeout=240)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]
