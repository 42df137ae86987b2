"""GPU tests of the reference-harness drop-in: every reference case through
every provider the reference allows for it, bound with Harness.bind and
launched through the returned closure, must equal the oracle bit for bit
(the reference's correctness runner, bench_welmv4_inplace_rope_npu.py:1524-1607,
checks each provider against the same oracle); misuse raises as in
Harness.bind (bench_welmv4_inplace_rope_npu.py:1177-1180, 1208-1213, 1268-1271)."""

from __future__ import annotations

import pytest
import torch

from oracle import rope_oracle
from testfiles_b200 import harness, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
CASES = {c.name: c for c in workloads.reference_cases()}
PAIRS = [(name, p) for name in sorted(CASES) for p in harness.providers_for_case(CASES[name])]


@pytest.fixture(scope="module")
def rig():
    return harness.Harness(DEV)


@pytest.mark.parametrize("name,provider", PAIRS)
def test_every_reference_case_through_every_provider(rig, name, provider):
    case = CASES[name]
    inp = workloads.make_inputs(case, "cpu")
    assert torch.equal(inp.cache, rig.cache.cpu()), "the harness cache is the reference's"
    dev = inp.to(DEV)
    launch = rig.bind(provider, case, dev.query, dev.key, dev.positions, dev.last_index, dev.segment_tile_starts)
    launch()
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    assert torch.equal(dev.query.cpu().view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(dev.key.cpu().view(torch.int16), k_ref.view(torch.int16))


def test_bind_rejects_what_the_reference_rejects(rig):
    def args(name):
        inp = workloads.make_inputs(CASES[name], "cpu").to(DEV)
        return CASES[name], inp

    case, inp = args("prefill_m128")
    with pytest.raises(ValueError, match="mirror_contiguous requires"):
        rig.bind("mirror_contiguous", case, inp.query, inp.key, inp.positions, inp.last_index, None)
    with pytest.raises(KeyError):
        rig.bind("no_such_provider", case, inp.query, inp.key, inp.positions, None, None)
    seg_mirror = next(n for n in CASES if CASES[n].is_segmented_mirror)
    case, inp = args(seg_mirror)
    with pytest.raises(ValueError, match="requires last_index and segment_tile_starts"):
        rig.bind("mirror_segmented", case, inp.query, inp.key, inp.positions, inp.last_index, None)
    with pytest.raises(ValueError, match="unsupported segmented mirror provider"):
        rig.bind("candidate", case, inp.query, inp.key, inp.positions, inp.last_index, inp.segment_tile_starts)
    seg = next(n for n in CASES if CASES[n].phase == "segmented_prefill")
    case, inp = args(seg)
    with pytest.raises(ValueError, match="segmented prefill requires segment_tile_starts"):
        rig.bind("segmented_prefill", case, inp.query, inp.key, inp.positions, None, None)
    with pytest.raises(ValueError, match="unsupported segmented provider"):
        rig.bind("baseline", case, inp.query, inp.key, inp.positions, None, inp.segment_tile_starts)
    assert rig.metadata()["num_q_heads"] == 6 and rig.metadata()["device_name"]


def test_bound_closures_replay_in_a_cuda_graph(rig):
    case = CASES["prefill_m2048"]
    inp = workloads.make_inputs(case, "cpu")
    dev = inp.to(DEV)
    launch = rig.bind("candidate", case, dev.query, dev.key, dev.positions, dev.last_index, dev.segment_tile_starts)
    launch()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch()
    graph.replay()
    torch.cuda.synchronize()
    # the eager launch and the replay each rotate once (capturing runs nothing)
    q1, k1 = rope_oracle.reference_outputs(inp.query, inp.key, inp.positions, inp.last_index, inp.cache)
    q2, k2 = rope_oracle.reference_outputs(q1, k1, inp.positions, inp.last_index, inp.cache)
    assert torch.equal(dev.query.cpu().view(torch.int16), q2.view(torch.int16))
    assert torch.equal(dev.key.cpu().view(torch.int16), k2.view(torch.int16))
