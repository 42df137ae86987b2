"""Pin the oracle (and the seeded input generators) against the reference.

The fixtures in tests/golden were produced by the reference's own
``make_cos_sin_cache`` / ``make_inputs`` / ``reference_outputs``
(bench_welmv4_inplace_rope_npu.py:1391-1521) by tests/golden/gen_golden.py.
Here the restated oracle must reproduce every output digest bit for bit,
and ``testfiles_b200.workloads`` must reproduce every input digest.  The
plain-C restatement (oracle/rope_oracle.c, through oracle/c_oracle.py) is held
to the same digests and to the reference's tile tables.
"""

from __future__ import annotations

import pytest
import torch

from conftest import digest
from oracle import c_oracle, rope_oracle
from testfiles_b200 import workloads

CASES = {c.name: c for c in workloads.reference_cases() + workloads.baseline_cases()}


def test_catalogue_matches_fixtures(golden_outputs):
    ref_names = {n for n, r in golden_outputs.items() if r["flavour"] == "reference"}
    assert len(ref_names) == 193
    assert {c.name for c in workloads.reference_cases()} == ref_names
    assert set(golden_outputs) == set(CASES)
    for name, rec in golden_outputs.items():
        case = CASES[name]
        assert (case.phase, case.n_tokens, case.batch_size) == (rec["phase"], rec["n_tokens"], rec["batch_size"])


def test_cache_restatement_matches_reference(golden_outputs):
    ref_digest = golden_outputs["prefill_m128"]["cache"]
    assert digest(rope_oracle.make_cos_sin_cache(32768, 100000.0)) == ref_digest
    assert digest(workloads.make_cos_sin_cache(32768, 100000.0)) == ref_digest
    base_digest = golden_outputs["b_prefill_m8192"]["cache"]
    assert digest(rope_oracle.make_cos_sin_cache(16384, 10000.0)) == base_digest


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_reproduces_reference(name, golden_outputs):
    rec = golden_outputs[name]
    case = CASES[name]
    inp = workloads.make_inputs(case, "cpu")
    got_inputs = {
        "query": digest(inp.query), "key": digest(inp.key), "positions": digest(inp.positions),
        "last_index": digest(inp.last_index), "segment_tile_starts": digest(inp.segment_tile_starts),
    }
    assert got_inputs == rec["inputs"], "seeded inputs differ from the reference's generators"
    if digest(inp.cache) != rec["cache"]:
        pytest.skip("this host's cos/sin differ in the last bit from the fixture host's")
    q_out, k_out = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert digest(q_out) == rec["outputs"]["query"]
    assert digest(k_out) == rec["outputs"]["key"]
    q_c, k_c = c_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert digest(q_c) == rec["outputs"]["query"], "C oracle differs from the reference"
    assert digest(k_c) == rec["outputs"]["key"], "C oracle differs from the reference"


def test_oracle_tile_builder_matches_reference_tables(tile_tables):
    assert len(tile_tables) == 13
    for name, rec in tile_tables.items():
        lens = rec["segment_lens"]
        assert rope_oracle.build_tile_starts(lens) == rec["segment_tile_starts"], name
        if rec["last_index"] is not None:
            assert rope_oracle.make_last_index(sum(lens), len(lens), lens) == rec["last_index"], name
        assert workloads.tile_starts_for(tuple(lens)) == rec["segment_tile_starts"], name
        assert c_oracle.build_tiles(lens) == rec["segment_tile_starts"], name


def test_oracle_uneven_lengths():
    assert rope_oracle.make_uneven_segment_lens(16384, 128) == workloads.reference_uneven_lens(16384, 128)
    lens = workloads.seeded_uneven_lens(9616, 128, 5)
    assert sum(lens) == 9616 and min(lens) >= 1 and len(lens) == 128


def test_oracle_legacy_last_index():
    assert rope_oracle.make_last_index(8192, 4) == [2047, 4095, 6143, 8191]
    assert rope_oracle.make_last_index(3, 8) == [0, 0, 0, 0, 0, 1, 1, 2]


def test_tiled_oracle_equals_full_oracle_for_wellformed_tables():
    case = workloads.find_case("segmented_m4096_b8_aligned")
    inp = workloads.make_inputs(case, "cpu")
    full = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, None, inp.cache)
    tiled = rope_oracle.tiled_outputs(inp.query, inp.key, inp.positions, inp.cache, inp.num_work_tiles, 1,
                                      inp.segment_tile_starts.tolist())
    assert torch.equal(full[0], tiled[0]) and torch.equal(full[1], tiled[1])


def test_rotated_tokens_caps_tiles_at_64():
    # a 100-token tile rotates only its first 64 tokens (reference masking rule)
    assert rope_oracle.rotated_tokens(120, 2, 1, [0, 100, 120]) == list(range(64)) + list(range(100, 120))
    assert rope_oracle.rotated_tokens(130, 2, 0) == list(range(128))


def test_position_zero_is_identity():
    cache = rope_oracle.make_cos_sin_cache(8, 10000.0)
    x = torch.randn(5, 6, 256, dtype=torch.bfloat16)
    out = rope_oracle.apply_reference(x, torch.zeros(5, dtype=torch.int64), cache)
    assert torch.equal(out, x)


def test_c_oracle_matches_torch_oracle_on_edge_values():
    """NaN / Inf / subnormal / out-of-range positions: the C restatement and
    the torch restatement agree bit for bit (bad rows are left unrotated)."""
    g = torch.Generator().manual_seed(7)
    cache = rope_oracle.make_cos_sin_cache(64, 10000.0)
    x = torch.randn(40, 3, 256, generator=g).to(torch.bfloat16)
    bits = x.view(torch.int16)
    bits[0, 0, 192:200] = torch.tensor([0x7FC0, 0x7F80, -128, 0x0001, -32767, 0x7F7F, -129, 0x7F81], dtype=torch.int16)
    bits[1, 2, 224:256] = 0x0001  # subnormal x2
    pos = torch.randint(0, 64, (40,), generator=g)
    pos[5] = 63
    out_t = rope_oracle.apply_reference(x, pos, cache)
    out_c = c_oracle.apply(x, pos, cache)
    # a rotated NaN's payload is not pinned (torch's vectorised CPU conversion
    # writes 0xFFFF, its scalar one 0x7FC0): NaN must meet NaN, the rest bits
    nan = torch.isnan(out_t)
    assert nan.any() and torch.equal(nan, torch.isnan(out_c))
    assert torch.equal(out_t.view(torch.int16)[~nan], out_c.view(torch.int16)[~nan])
    bad = pos.clone()
    bad[3], bad[4] = -1, 64
    out_b = c_oracle.apply(x, bad, cache)
    keep = torch.ones(40, dtype=torch.bool)
    keep[3:5] = False
    assert torch.equal(out_b[keep].view(torch.int16), out_c[keep].view(torch.int16))
    assert torch.equal(out_b[3:5].view(torch.int16), x[3:5].view(torch.int16))


def test_c_oracle_tile_builder_edge_lengths():
    for lens in ([], [0], [0, 0, 5], [64], [65, 0, 128, 1], [1] * 70, [4096, 3]):
        assert c_oracle.build_tiles(lens) == rope_oracle.build_tile_starts(lens), lens


def test_c_and_torch_oracles_agree_on_random_inputs():
    """Property check beyond the fixtures: random row and head counts,
    positions over the whole cache (both ends included), values spanning
    several binades.  NaN cannot arise from finite inputs here."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    cache = rope_oracle.make_cos_sin_cache(512, 10000.0)

    @settings(max_examples=60, deadline=None)
    @given(rows=st.integers(1, 40), heads=st.sampled_from([1, 6]), seed=st.integers(0, 2**31 - 1),
           scale=st.sampled_from([1e-3, 1.0, 300.0]))
    def check(rows, heads, seed, scale):
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(rows, heads, 256, generator=g) * scale).to(torch.bfloat16)
        pos = torch.randint(0, 512, (rows,), generator=g)
        pos[0] = 0
        pos[-1] = 511
        want = rope_oracle.apply_reference(x, pos, cache)
        got = c_oracle.apply(x, pos, cache)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))

    check()
