#!/usr/bin/env python3
"""Correctness records: every catalogue case through every entry, on a GPU,
checked against the oracle.

    python tests/parity_records.py [--cases reference,baseline] [--json out.jsonl] [--csv out.csv]

One record per case x entry.  Each has the form of the reference benchmark's
correctness record (bench_welmv4_inplace_rope_npu.py:1573-1605): record_type
"correctness", the case fields, variant, status, atol/rtol, max_abs_q and
max_abs_k.  Each also states what this build claims about its results:

* the BF16 ulp distance of every rotated lane from the oracle, as a histogram
  (0, 1, more than 1);
* whether lanes 0..191 of Q and K are unchanged (the reference's prefix
  check, bench_welmv4_inplace_rope_npu.py:1577-1581);
* whether the outputs are bit-exact.

status is PASS when the prefix is unchanged and no rotated lane is more than
1 ulp away (the bar this port is held to), FAIL otherwise.

Which entries run:

* Reference cases go through every provider the reference binds for them
  (Harness.bind, bench_welmv4_inplace_rope_npu.py:1088-1100, 1121-1388).
* Benchmark configurations (another cos/sin cache) go through the production
  entry welmv4_inplace_rope_npu.  Segmented KV-mirror configurations also go
  through rope_mirror_from_lens.

This is test infrastructure: it imports the oracle.  The GPU test
tests/test_gpu_records.py runs it over every case.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Iterable, Optional

import torch

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from oracle import rope_oracle  # noqa: E402
from testfiles_b200 import harness, launcher, ops, workloads  # noqa: E402

ROPE_LANE0 = 192
ATOL = 0.0
RTOL = 0.0


def ordered_bf16(t: torch.Tensor) -> torch.Tensor:
    """BF16 bits mapped to integers that order like the values (so the
    difference of two is their distance in ulps); -0 and +0 both map to 0."""
    u = t.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    return torch.where(u >= 0x8000, 0x8000 - u, u)


def compare(out: torch.Tensor, ref: torch.Tensor, before: torch.Tensor) -> dict:
    """Max-abs difference, ulp histogram of the rotated lanes, prefix check."""
    out, ref, before = out.cpu(), ref.cpu(), before.cpu()
    rot_out, rot_ref = out[..., ROPE_LANE0:], ref[..., ROPE_LANE0:]
    ulp = (ordered_bf16(rot_out) - ordered_bf16(rot_ref)).abs()
    return {
        "max_abs": float((out.float() - ref.float()).abs().max()) if out.numel() else 0.0,
        "ulp0": int((ulp == 0).sum()),
        "ulp1": int((ulp == 1).sum()),
        "ulp_gt1": int((ulp > 1).sum()),
        "max_ulp": int(ulp.max()) if ulp.numel() else 0,
        "prefix_equal": bool(torch.equal(out[..., :ROPE_LANE0].view(torch.int16),
                                         before[..., :ROPE_LANE0].view(torch.int16))),
        "bit_exact": bool(torch.equal(out.view(torch.int16), ref.view(torch.int16))),
    }


def record(case: workloads.Case, variant: str, q_out, k_out, q_ref, k_ref, q_in, k_in) -> dict:
    cq, ck = compare(q_out, q_ref, q_in), compare(k_out, k_ref, k_in)
    ok = cq["prefix_equal"] and ck["prefix_equal"] and cq["max_ulp"] <= 1 and ck["max_ulp"] <= 1
    return {
        "record_type": "correctness",
        **launcher.case_fields(case),
        "variant": variant,
        "status": "PASS" if ok else "FAIL",
        "atol": ATOL,
        "rtol": RTOL,
        "max_abs_q": cq["max_abs"],
        "max_abs_k": ck["max_abs"],
        "max_ulp_q": cq["max_ulp"],
        "max_ulp_k": ck["max_ulp"],
        "ulp_hist_q": {"0": cq["ulp0"], "1": cq["ulp1"], ">1": cq["ulp_gt1"]},
        "ulp_hist_k": {"0": ck["ulp0"], "1": ck["ulp1"], ">1": ck["ulp_gt1"]},
        "prefix_equal_q": cq["prefix_equal"],
        "prefix_equal_k": ck["prefix_equal"],
        "bit_exact": cq["bit_exact"] and ck["bit_exact"],
    }


def case_records(case: workloads.Case, device: torch.device, rig: Optional[harness.Harness]) -> list[dict]:
    inp = workloads.make_inputs(case, "cpu")
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    out = []
    if case.flavour == "reference":
        for provider in harness.providers_for_case(case):
            d = inp.to(device)
            rig.bind(provider, case, d.query, d.key, d.positions, d.last_index, d.segment_tile_starts)()
            torch.cuda.synchronize(device)
            out.append(record(case, provider, d.query, d.key, q_ref, k_ref, inp.query, inp.key))
        return out
    d = inp.to(device)
    ops.welmv4_inplace_rope_npu(d.query, d.key, d.positions, d.cache, d.last_index, d.segment_tile_starts)
    torch.cuda.synchronize(device)
    out.append(record(case, "welmv4_inplace_rope_npu", d.query, d.key, q_ref, k_ref, inp.query, inp.key))
    if case.is_segmented_mirror:
        d = inp.to(device)
        lens = torch.tensor(case.segment_lens, dtype=torch.int64, device=device)
        ops.rope_mirror_from_lens(d.query, d.key, d.positions, d.cache, lens)
        torch.cuda.synchronize(device)
        out.append(record(case, "rope_mirror_from_lens", d.query, d.key, q_ref, k_ref, inp.query, inp.key))
    return out


def select(spec: str) -> list[workloads.Case]:
    groups = {"reference": workloads.reference_cases(), "baseline": workloads.baseline_cases()}
    cases: list[workloads.Case] = []
    for item in spec.split(","):
        item = item.strip()
        if item:
            cases.extend(groups[item] if item in groups else [workloads.find_case(item)])
    return cases


def run(cases: Iterable[workloads.Case], device: torch.device) -> list[dict]:
    rig = harness.Harness(device)
    records: list[dict] = []
    for case in cases:
        records.extend(case_records(case, device, rig))
    return records


def summary(records: list[dict]) -> dict:
    return {
        "records": len(records),
        "cases": len({r["case"] for r in records}),
        "pass": sum(r["status"] == "PASS" for r in records),
        "bit_exact": sum(r["bit_exact"] for r in records),
        "max_abs_q": max((r["max_abs_q"] for r in records), default=0.0),
        "max_abs_k": max((r["max_abs_k"] for r in records), default=0.0),
        "max_ulp": max((max(r["max_ulp_q"], r["max_ulp_k"]) for r in records), default=0),
        "rotated_lanes_checked": sum(sum(r["ulp_hist_q"].values()) + sum(r["ulp_hist_k"].values())
                                     for r in records),
        "prefix_equal": sum(r["prefix_equal_q"] and r["prefix_equal_k"] for r in records),
    }


def main(argv: Optional[list[str]] = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--cases", default="reference,baseline", help="case names or groups (reference, baseline)")
    parser.add_argument("--device", default="cuda:0")
    parser.add_argument("--json", default=None, help="write the records as JSON lines here")
    parser.add_argument("--csv", default=None, help="write the records as one CSV table here")
    args = parser.parse_args(argv)
    if not torch.cuda.is_available():
        print("parity_records needs a CUDA device", file=sys.stderr)
        return 2
    device = torch.device(args.device)
    torch.cuda.set_device(device)
    records = run(select(args.cases), device)
    if args.json:
        with open(args.json, "w") as fh:
            for rec in records:
                fh.write(json.dumps(rec) + "\n")
    if args.csv:
        launcher.write_csv(records, args.csv)
    print(json.dumps(summary(records)))
    return 0 if all(r["status"] == "PASS" for r in records) else 1


if __name__ == "__main__":
    raise SystemExit(main())
