"""GPU tests of the profiling launcher: its records carry the fields the
profiles quote, with sane values (small cases, few replays)."""

from __future__ import annotations

import json

import pytest
import torch

import testfiles_b200 as welm
from testfiles_b200 import launcher, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.mark.parametrize("name", ["b_prefill_m577", "b_mirror_segmented_n8192_bs4_uneven"])
def test_time_case_with_copy_ceiling(name):
    case = workloads.find_case(name)
    rec = launcher.time_case(case, DEV, trials=3, graph_launches=8, replays=5, copy_ceiling=True)
    assert rec["record_type"] == "timing" and rec["case"] == name
    assert rec["us_per_launch"] > 0 and rec["same_size_copy_us"] > 0
    assert rec["bytes_per_launch"] == workloads.min_bytes(case)
    assert 0 < rec["frac_of_same_size_copy"] < 10
    assert rec["gb_s"] == pytest.approx(rec["bytes_per_launch"] / (rec["us_per_launch"] * 1e3), rel=0.01)
    assert set(rec["clocks"]) >= {"sm_mhz", "sm_max_mhz", "reasons", "samples"}
    assert rec["stream_copy_us"] > 0 and rec["frac_of_stream_copy"] > 0
    assert ("slice_floor_us" in rec) == (not case.is_mirror)
    json.dumps(rec)


def test_launch_records_and_json_sink(tmp_path):
    out = tmp_path / "records.jsonl"
    recs = launcher.run(launcher.select_cases("b_prefill_m577"), DEV, False, 2, str(out))
    assert recs[0]["record_type"] == "launch" and recs[0]["kernel_name"] == "rope_ordinary_head_kernel"
    assert json.loads(out.read_text().splitlines()[0])["case"] == "b_prefill_m577"


@pytest.mark.parametrize("transport", ["mapped", "staged"])
def test_time_host_case(transport):
    case = workloads.find_case("b_prefill_m577")
    rec = launcher.time_host_case(case, DEV, transport, trials=2, calls=3)
    assert rec["record_type"] == "host_timing" and rec["transport"] == transport
    assert rec["us_per_call"] > 0 and rec["d2h_bytes_per_call"] == 577 * 7 * 128
    with pytest.raises(ValueError):
        launcher.time_host_case(workloads.find_case("b_mirror_contiguous_n8192"), DEV, transport)


def test_time_kv_write_record():
    rec = launcher.time_kv_write(1000, 7, DEV, trials=2, graph_launches=4, replays=3, sets=2)
    assert rec["us_per_launch"] > 0 and rec["bytes_per_launch"] == launcher.kv_write_bytes(1000, 7)
    assert rec["same_size_copy_us"] > 0
    assert launcher.time_kv_write(500, 3, DEV, iters=2)["record_type"] == "launch"


def test_time_fused_qkv_record():
    rec = launcher.time_fused_qkv(1000, DEV, trials=2, graph_launches=4, replays=3, sets=2)
    assert rec["path"] == "fused_qkv_strided" and rec["bytes_per_launch"] == 2056 * 1000
    assert rec["us_per_launch"] > 0 and rec["copy_then_rope_us"] > 0
    assert rec["saved_us"] == pytest.approx(rec["copy_then_rope_us"] - rec["us_per_launch"], abs=2e-3)
    json.dumps(rec)


def test_ceiling_kernels_copy_exactly_and_leave_slices_unchanged():
    g = torch.Generator(device=DEV).manual_seed(5)
    # one vector per thread; four per thread in one wave; four per thread over
    # two rounds with a remainder
    for size, nbytes in ((1 << 20, (1 << 20) - 4096), (8 << 20, 8 << 20), ((20 << 20) + 4096, (20 << 20) + 48)):
        src = torch.randint(0, 256, (size,), dtype=torch.uint8, device=DEV, generator=g)
        dst = torch.zeros_like(src)
        launcher.ceiling_copy(dst, src, nbytes)
        torch.cuda.synchronize()
        assert torch.equal(dst[:nbytes], src[:nbytes]), nbytes
        assert int(dst[nbytes:].count_nonzero()) == 0, nbytes  # nothing past nbytes
    with pytest.raises(ValueError):
        launcher.ceiling_copy(dst, src, size + 16)

    m = 3001
    qkv = torch.randn((m, 8 * 256), device=DEV, generator=g).to(torch.bfloat16)
    before = qkv.clone()
    launcher.ceiling_slices(qkv[:, :1536].view(m, 6, 256), qkv[:, 1536:1792].view(m, 1, 256))
    torch.cuda.synchronize()
    assert torch.equal(qkv.view(torch.int16), before.view(torch.int16))
    for rows in (3001, 5000):  # one head per thread up to 3328 tokens, seven above
        q = torch.randn((rows, 6, 256), device=DEV, generator=g).to(torch.bfloat16)
        k = torch.randn((rows, 1, 256), device=DEV, generator=g).to(torch.bfloat16)
        q0, k0 = q.clone(), k.clone()
        launcher.ceiling_slices(q, k)
        torch.cuda.synchronize()
        assert torch.equal(q.view(torch.int16), q0.view(torch.int16)), rows
        assert torch.equal(k.view(torch.int16), k0.view(torch.int16)), rows


@pytest.mark.parametrize("rows,fused,ctas,stages", [(16384, False, 0, 6), (1000, True, 148, 4), (7, False, 5, 2),
                                                    (1000, False, 3, 2), (3001, True, 0, 6)])
def test_tma_ceiling_leaves_slices_and_neighbours_unchanged(rows, fused, ctas, stages):
    """The TMA-staged mover rewrites the rope slices with themselves; rows
    past N (outside its tensor maps) and the other lanes stay untouched, and
    no barrier wait gives up."""
    g = torch.Generator(device=DEV).manual_seed(rows + stages)
    extra = 40
    if fused:
        qkv = torch.randn((rows + extra, 8 * 256), device=DEV, generator=g).to(torch.bfloat16)
        q, k = qkv[:rows, :1536].view(rows, 6, 256), qkv[:rows, 1536:1792].view(rows, 1, 256)
        stores = [qkv]
    else:
        qb = torch.randn((rows + extra, 6, 256), device=DEV, generator=g).to(torch.bfloat16)
        kb = torch.randn((rows + extra, 1, 256), device=DEV, generator=g).to(torch.bfloat16)
        q, k = qb[:rows], kb[:rows]
        stores = [qb, kb]
    before = [t.clone() for t in stores]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    launcher.ceiling_tma_slices(q, k, ctas, stages, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for t, t0 in zip(stores, before):
        assert torch.equal(t.view(torch.int16), t0.view(torch.int16))
    with pytest.raises(welm.WelmRopeError):
        launcher.ceiling_tma_slices(q, k, ctas, 3)


def test_tma_floor_timing():
    bufs = [(torch.randn((4096, 6, 256), device=DEV).to(torch.bfloat16),
             torch.randn((4096, 1, 256), device=DEV).to(torch.bfloat16)) for _ in range(2)]
    us = launcher.tma_floor_us(bufs, DEV, stages=4, trials=2, graph_launches=8, replays=2)
    assert 0.0 < us < 1000.0


def test_gather_ceiling_reads_without_writing():
    """welm_rope_ceiling_gather runs the op's position and cos/sin gather alone:
    it returns without error on every launch shape, rejects bad tensors on the
    host, and writes nothing (its sink is never set for a real cache)."""
    cache = workloads.make_cos_sin_cache(16384, 10000.0, device=DEV)
    for m in (1, 100, 5000, 16384, 40000):  # warp-sized CTAs, 128-thread CTAs, and looping threads
        pos = (torch.arange(m, device=DEV, dtype=torch.int64) * 7) % 16384
        pos_before, cache_before = pos.clone(), cache.clone()
        launcher.ceiling_gather(pos, cache)
        torch.cuda.synchronize()
        assert torch.equal(pos, pos_before) and torch.equal(cache, cache_before), m
    with pytest.raises(TypeError):
        launcher.ceiling_gather(pos.to(torch.int32), cache)
    with pytest.raises(ValueError):
        launcher.ceiling_gather(pos[::2], cache)
