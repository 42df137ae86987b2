"""CPU checks of the correctness-record arithmetic in tests/parity_records.py:
BF16 ulp distances, the prefix check and the PASS rule."""

from __future__ import annotations

import torch

import parity_records as pr


def bf16(bits: list[int]) -> torch.Tensor:
    return torch.tensor(bits, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)


def test_ulp_distance_follows_value_order():
    one, next_up = bf16([0x3F80]), bf16([0x3F81])          # 1.0 and the next BF16 above it
    minus_one, next_down = bf16([0xBF80]), bf16([0xBF81])  # -1.0 and the next BF16 below it
    pos0, neg0 = bf16([0x0000]), bf16([0x8000])
    tiny_pos, tiny_neg = bf16([0x0001]), bf16([0x8001])
    d = lambda a, b: int((pr.ordered_bf16(a) - pr.ordered_bf16(b)).abs())  # noqa: E731
    assert d(one, next_up) == 1 and d(minus_one, next_down) == 1
    assert d(pos0, neg0) == 0
    assert d(tiny_pos, tiny_neg) == 2  # across zero: -min, 0, +min
    assert d(one, minus_one) == 2 * 0x3F80


def test_compare_counts_ulps_and_checks_the_prefix():
    g = torch.Generator().manual_seed(0)
    ref = torch.randn((3, 6, 256), generator=g).to(torch.bfloat16)
    before = ref.clone()
    out = ref.clone()
    bits = out.view(torch.int16)
    bits[0, 0, 200] += 1   # one rotated lane 1 ulp off
    bits[1, 2, 250] += 3   # one rotated lane 3 ulps off
    c = pr.compare(out, ref, before)
    assert c["ulp1"] == 1 and c["ulp_gt1"] == 1 and c["max_ulp"] == 3
    assert c["ulp0"] == 3 * 6 * 64 - 2
    assert c["prefix_equal"] and not c["bit_exact"] and c["max_abs"] > 0
    bits[2, 5, 10] += 1    # a lane the op must never write
    assert not pr.compare(out, ref, before)["prefix_equal"]


def test_pass_rule_is_one_ulp_and_an_untouched_prefix():
    from testfiles_b200 import workloads

    case = workloads.find_case("b_prefill_m128")
    g = torch.Generator().manual_seed(1)
    q = torch.randn((4, 6, 256), generator=g).to(torch.bfloat16)
    k = torch.randn((4, 1, 256), generator=g).to(torch.bfloat16)
    exact = pr.record(case, "x", q, k, q, k, q, k)
    assert exact["status"] == "PASS" and exact["bit_exact"] and exact["max_abs_q"] == 0.0
    q1 = q.clone()
    q1.view(torch.int16)[0, 0, 255] += 1
    assert pr.record(case, "x", q1, k, q, k, q, k)["status"] == "PASS"
    q2 = q.clone()
    q2.view(torch.int16)[0, 0, 255] += 2
    assert pr.record(case, "x", q2, k, q, k, q, k)["status"] == "FAIL"
    assert exact["record_type"] == "correctness" and exact["case"] == "b_prefill_m128"
