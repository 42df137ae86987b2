"""GPU tests of the profiling launcher: its records carry the fields the
profiles quote, with sane values (small cases, few replays)."""

from __future__ import annotations

import json

import pytest
import torch

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
    json.dumps(rec)


def test_launch_records_and_json_sink(tmp_path):
    out = tmp_path / "records.jsonl"
    recs = launcher.run(launcher.select_cases("b_prefill_m577"), DEV, False, 2, str(out))
    assert recs[0]["record_type"] == "launch" and recs[0]["kernel_name"] == "rope_ordinary_kernel"
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
