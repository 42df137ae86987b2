"""GPU tests of the KV-mirror pass fused with the paged KV-cache write and
the Q last-row extraction (rope_mirror_kv_write), against an oracle built
from the reference's apply_reference: bit for bit, untouched cache rows stay
untouched, inputs are not modified."""

from __future__ import annotations

import pytest
import torch

from oracle import rope_oracle
import testfiles_b200 as welm
from testfiles_b200 import _native, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
SENTINEL = -3.0


def make_case(n: int, bs: int, num_blocks: int, block_size: int, seed: int, pad_every: int = 0, layout="nhd"):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn((n, 8 * 256), dtype=torch.bfloat16, generator=g)  # fused projection output
    positions = torch.randint(0, 4096, (n,), generator=g, dtype=torch.int64)
    lens = workloads.seeded_uneven_lens(n, bs, seed)
    last_index = torch.tensor(lens).cumsum(0) - 1
    slots = torch.randperm(num_blocks * block_size, generator=g)[:n].to(torch.int64)
    if pad_every:
        slots[::pad_every] = -1
    shape = (num_blocks, block_size, 1, 256) if layout == "nhd" else (num_blocks, 1, block_size, 256)
    cache_k = torch.full(shape, SENTINEL, dtype=torch.bfloat16)
    cache_v = torch.full(shape, SENTINEL, dtype=torch.bfloat16)
    cos_sin = workloads.make_cos_sin_cache(4096, 10000.0)
    return qkv, positions, last_index, slots, cache_k, cache_v, cos_sin


def expected(qkv, positions, last_index, slots, cache_k, cache_v, cos_sin):
    n = qkv.shape[0]
    q = qkv[:, :1536].reshape(n, 6, 256)
    k = qkv[:, 1536:1792].reshape(n, 1, 256)
    v = qkv[:, 1792:].reshape(n, 1, 256)
    q_out = rope_oracle.apply_reference(q[last_index], positions[last_index], cos_sin)
    k_rot = rope_oracle.apply_reference(k, positions, cos_sin)
    ck = cache_k.clone().reshape(-1, 256)
    cv = cache_v.clone().reshape(-1, 256)
    keep = slots >= 0
    ck[slots[keep]] = k_rot[keep].reshape(-1, 256)
    cv[slots[keep]] = v[keep].reshape(-1, 256)
    return q_out, ck.reshape(cache_k.shape), cv.reshape(cache_v.shape)


@pytest.mark.parametrize("n,bs,blocks,bsz,pad,layout", [
    (3000, 7, 60, 64, 0, "nhd"), (16384, 128, 300, 64, 0, "nhd"), (1000, 1, 40, 32, 9, "hnd"), (5, 5, 1, 16, 2, "nhd"),
])
def test_kv_write_matches_oracle(n, bs, blocks, bsz, pad, layout):
    qkv, positions, last_index, slots, cache_k, cache_v, cos_sin = make_case(n, bs, blocks, bsz, n + bs, pad, layout)
    want_q, want_k, want_v = expected(qkv, positions, last_index, slots, cache_k, cache_v, cos_sin)
    d = qkv.to(DEV)
    before = d.clone()
    q_out = torch.zeros((bs, 6, 256), dtype=torch.bfloat16, device=DEV)
    ck, cv = cache_k.to(DEV), cache_v.to(DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    welm.rope_mirror_kv_write(d[:, :1536].view(n, 6, 256), q_out, d[:, 1536:1792].view(n, 1, 256),
                              d[:, 1792:].view(n, 1, 256), positions.to(DEV), cos_sin.to(DEV), last_index.to(DEV),
                              slots.to(DEV), ck, cv, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(q_out.cpu().view(torch.int16), want_q.view(torch.int16))
    assert torch.equal(ck.cpu().view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(cv.cpu().view(torch.int16), want_v.view(torch.int16))
    assert torch.equal(d, before)  # q, k and v are read only


def test_kv_write_without_v_and_bad_slots():
    n, bs = 400, 3
    qkv, positions, last_index, slots, cache_k, cache_v, cos_sin = make_case(n, bs, 10, 64, 11)
    slots[[5, 77]] = torch.tensor([640, 10_000])  # past the 640 slots
    good = slots < 640
    want_q, want_k, _ = expected(qkv, positions, last_index, torch.where(good, slots, -1), cache_k, cache_v, cos_sin)
    d = qkv.to(DEV)
    q_out = torch.zeros((bs, 6, 256), dtype=torch.bfloat16, device=DEV)
    ck = cache_k.to(DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    welm.rope_mirror_kv_write(d[:, :1536].view(n, 6, 256), q_out, d[:, 1536:1792].view(n, 1, 256), None,
                              positions.to(DEV), cos_sin.to(DEV), last_index.to(DEV), slots.to(DEV), ck, None,
                              status=status)
    torch.cuda.synchronize()
    assert status.item() == _native.DEV_BAD_SLOT
    assert torch.equal(q_out.cpu().view(torch.int16), want_q.view(torch.int16))
    assert torch.equal(ck.cpu().view(torch.int16), want_k.view(torch.int16))


def test_kv_write_graph_replays_with_changing_positions():
    """The producer (a copy of new positions and activations) and the fused
    write in one CUDA graph: each replay's pre-wait position hints are stale
    on purpose, and every replay must still equal the oracle."""
    n, bs = 3000, 7
    qkv, positions, last_index, slots, cache_k, cache_v, cos_sin = make_case(n, bs, 60, 64, 5)
    qkv_src, pos_src = qkv.to(DEV), positions.to(DEV)
    d, pos = torch.empty_like(qkv_src), torch.empty_like(pos_src)
    q_out = torch.zeros((bs, 6, 256), dtype=torch.bfloat16, device=DEV)
    ck, cv = cache_k.to(DEV), cache_v.to(DEV)
    dev_cache, dev_last, dev_slots = cos_sin.to(DEV), last_index.to(DEV), slots.to(DEV)

    def step():
        d.copy_(qkv_src)
        pos.copy_(pos_src)
        welm.rope_mirror_kv_write(d[:, :1536].view(n, 6, 256), q_out, d[:, 1536:1792].view(n, 1, 256),
                                  d[:, 1792:].view(n, 1, 256), pos, dev_cache, dev_last, dev_slots, ck, cv)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for seed in (1, 2, 3):
        g = torch.Generator().manual_seed(seed)
        new_pos = torch.randint(0, 4096, (n,), generator=g, dtype=torch.int64)
        new_qkv = torch.randn((n, 8 * 256), generator=g).to(torch.bfloat16)
        pos_src.copy_(new_pos)
        qkv_src.copy_(new_qkv)
        graph.replay()
        torch.cuda.synchronize()
        want_q, want_k, want_v = expected(new_qkv, new_pos, last_index, slots, cache_k, cache_v, cos_sin)
        assert torch.equal(q_out.cpu().view(torch.int16), want_q.view(torch.int16)), seed
        assert torch.equal(ck.cpu().view(torch.int16), want_k.view(torch.int16)), seed
        assert torch.equal(cv.cpu().view(torch.int16), want_v.view(torch.int16)), seed
