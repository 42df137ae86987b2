"""The reference-harness drop-in (testfiles_b200.harness): provider tables
and per-case provider selection, restated from
bench_welmv4_inplace_rope_npu.py:922-935 and 1088-1100."""

from __future__ import annotations

from testfiles_b200 import harness, workloads


def test_provider_tables_match_the_reference():
    assert set(harness.PROVIDERS) == {"baseline", "candidate", "generic_prefill", "segmented_prefill",
                                      "mirror_contiguous", "mirror_segmented"}
    assert harness.DEFAULT_PROVIDERS == ("baseline", "candidate")
    assert harness.SEGMENTED_PROVIDERS == ("generic_prefill", "segmented_prefill")
    assert harness.CONTIGUOUS_MIRROR_PROVIDERS == ("baseline", "mirror_contiguous")
    assert harness.SEGMENTED_MIRROR_PROVIDERS == ("baseline", "mirror_segmented")
    assert harness.LEGACY_MIRROR_PROVIDERS == ("baseline",)


def test_providers_for_every_reference_case():
    expected = {
        "decode": ("baseline", "candidate"),
        "prefill": ("baseline", "candidate"),
        "segmented_prefill": ("generic_prefill", "segmented_prefill"),
        "prefill_mirror": ("baseline",),
        "prefill_mirror_contiguous": ("baseline", "mirror_contiguous"),
        "prefill_mirror_segmented": ("baseline", "mirror_segmented"),
    }
    cases = workloads.reference_cases() + workloads.baseline_cases()
    seen = set()
    for case in cases:
        assert harness.providers_for_case(case) == expected[case.phase], case.name
        seen.add(case.phase)
    assert seen == set(expected)


def test_case_properties():
    case = workloads.find_case("b_mirror_segmented_n16384_bs128_uneven")
    assert case.is_segmented_mirror and not case.is_contiguous_mirror and case.request_count == 128
    case = workloads.find_case("b_mirror_contiguous_n16384")
    assert case.is_contiguous_mirror and not case.is_segmented_mirror and case.request_count == 0
