"""CPU checks of the figures bench.py reports beside its timing: the
algorithmic byte count, the ncu traffic figure it reads from the committed
profile, the published figure behind vs_baseline, and the result-line
configuration."""

from __future__ import annotations

import importlib.util

from conftest import REPO
from testfiles_b200 import workloads


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_algorithmic_bytes_match_the_workload_model():
    bench = load_bench()
    case = workloads.find_case("b_prefill_m16384")
    assert bench.algorithmic_bytes(bench.TOKENS) == workloads.min_bytes(case) == 33_685_504


def test_traffic_figure_comes_from_the_committed_profile():
    bench = load_bench()
    traffic, source = bench.profiled_traffic()
    assert traffic is not None
    # DRAM bytes per launch close to the algorithmic reads (writes stay in L2)
    assert 19_000_000 <= traffic <= 19_100_000
    # the line says where the figure comes from: a separate capture, not this run
    assert "profiles/rope_ordinary_prefill_m16384.md" in source and "not measured by this run" in source


def test_vs_baseline_uses_the_published_figure():
    bench = load_bench()
    assert abs(bench.PUBLISHED_GBS - bench.algorithmic_bytes(bench.TOKENS) / 38.69e-6 / 1e9) < 1.0
    assert "38.69" in bench.PUBLISHED_SOURCE


def test_result_line_configuration():
    bench = load_bench()
    cfg = bench.workload_config(4)
    assert cfg["global_tokens"] == 4 * bench.TOKENS and cfg["parallelism"] == "request-sharded dp4"
    assert bench.BUFFER_SETS * bench.algorithmic_bytes(bench.TOKENS) > 2 * 126 * 1024 * 1024
    assert set(bench.OTHER_CONFIGS) <= {c.name for c in workloads.baseline_cases()}
