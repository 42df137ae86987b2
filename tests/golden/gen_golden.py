#!/usr/bin/env python3
"""Generate the golden fixtures from the reference's OWN Python code.

Run where the reference source tree is available, naming its directory
(or set WELM_ROPE_REFERENCE_DIR):

    python tests/golden/gen_golden.py --reference <reference checkout>

It imports ``bench_welmv4_inplace_rope_npu`` with an empty stand-in for the
Ascend-only ``torch_npu`` module (nothing of that module is used by the
functions called here), then, on the CPU:

* for every case of the reference catalogue: the reference's own
  ``make_cos_sin_cache``, ``make_inputs`` (seed 20260814) and
  ``reference_outputs``;
* for every benchmark ("baseline") configuration: inputs from
  ``testfiles_b200.workloads`` run through the reference's own
  ``reference_outputs``.

It writes SHA-256 digests of every input and output tensor to
``golden_outputs.json`` and the reference's segmented tile tables and
``last_index`` vectors verbatim to ``tile_tables.json``.  The fixtures are
small (digests, not tensors); the tests regenerate the seeded inputs, check
their digests, and compare output digests.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import platform
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def digest(t: torch.Tensor | None) -> str | None:
    if t is None:
        return None
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def load_reference(path: Path):
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    sys.path.insert(0, str(path))
    import bench_welmv4_inplace_rope_npu as ref  # noqa: E402

    return ref


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("WELM_ROPE_REFERENCE_DIR"),
                        help="directory of the reference checkout (default: $WELM_ROPE_REFERENCE_DIR)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("name the reference checkout with --reference or WELM_ROPE_REFERENCE_DIR")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = load_reference(Path(args.reference))
    sys.path.insert(0, str(REPO))
    from testfiles_b200 import workloads  # noqa: E402

    cpu = torch.device("cpu")
    ref_cache = ref.make_cos_sin_cache(cpu)
    records: dict[str, dict] = {}
    tables: dict[str, dict] = {}

    for case in ref.ALL_CASES:
        q, k, pos, last, starts = ref.make_inputs(case, cpu, 20260814)  # the CLI default seed
        q_out, k_out = ref.reference_outputs(q, k, pos, last, ref_cache)
        records[case.name] = {
            "flavour": "reference",
            "phase": case.phase,
            "n_tokens": case.n_tokens,
            "batch_size": case.batch_size,
            "cache": digest(ref_cache),
            "inputs": {"query": digest(q), "key": digest(k), "positions": digest(pos),
                       "last_index": digest(last), "segment_tile_starts": digest(starts)},
            "outputs": {"query": digest(q_out), "key": digest(k_out)},
        }
        if starts is not None:
            tables[case.name] = {
                "segment_lens": list(case.segment_lens),
                "segment_tile_starts": [int(v) for v in starts.tolist()],
                "last_index": None if last is None else [int(v) for v in last.tolist()],
            }

    for case in workloads.baseline_cases():
        inp = workloads.make_inputs(case, "cpu")
        q_out, k_out = ref.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
        records[case.name] = {
            "flavour": "baseline",
            "phase": case.phase,
            "n_tokens": case.n_tokens,
            "batch_size": case.batch_size,
            "segment_lens": list(case.segment_lens),
            "cache": digest(inp.cache),
            "inputs": {"query": digest(inp.query), "key": digest(inp.key), "positions": digest(inp.positions),
                       "last_index": digest(inp.last_index), "segment_tile_starts": digest(inp.segment_tile_starts)},
            "outputs": {"query": digest(q_out), "key": digest(k_out)},
        }

    meta = {
        "generator": "tests/golden/gen_golden.py",
        "source": "bench_welmv4_inplace_rope_npu.py make_cos_sin_cache / make_inputs / reference_outputs",
        "torch": torch.__version__,
        "python": platform.python_version(),
        "machine": platform.machine(),
    }
    (HERE / "golden_outputs.json").write_text(json.dumps({"meta": meta, "cases": records}, indent=1, sort_keys=True))
    (HERE / "tile_tables.json").write_text(json.dumps({"meta": meta, "cases": tables}, indent=1, sort_keys=True))
    print(f"wrote {len(records)} output records and {len(tables)} tile tables")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
