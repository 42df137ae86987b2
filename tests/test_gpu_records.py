"""Correctness records over every catalogue case (tests/parity_records.py):
every reference case through every provider the reference binds for it, and
every benchmark configuration through the production entry (segmented
mirrors also through rope_mirror_from_lens), each checked against the oracle.
Every record must PASS and be bit-exact: 0 ulp on every rotated lane, lanes
0..191 unchanged, max_abs_q = max_abs_k = 0."""

from __future__ import annotations

import json

import pytest
import torch

import parity_records as pr

pytestmark = pytest.mark.gpu


def test_every_case_and_entry_is_bit_exact(tmp_path):
    dev = torch.device("cuda:0")
    records = pr.run(pr.select("reference,baseline"), dev)
    s = pr.summary(records)
    assert s["cases"] == 193 + 213
    assert s["records"] >= s["cases"]
    bad = [(r["case"], r["variant"], r["max_ulp_q"], r["max_ulp_k"]) for r in records if not r["bit_exact"]]
    assert not bad, bad[:10]
    assert s["pass"] == s["records"] and s["prefix_equal"] == s["records"]
    assert s["max_abs_q"] == 0.0 and s["max_abs_k"] == 0.0 and s["max_ulp"] == 0
    out = tmp_path / "records.jsonl"
    out.write_text("".join(json.dumps(r) + "\n" for r in records))
    assert len(out.read_text().splitlines()) == len(records)
