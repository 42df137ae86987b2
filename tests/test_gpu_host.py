"""GPU tests of the host-memory entry (welmv4_inplace_rope_host) and the
rope-lane copy helper: results must equal the oracle bit for bit and lanes
0..191 of the host tensors must stay untouched."""

from __future__ import annotations

import pytest
import torch

from oracle import rope_oracle
from testfiles_b200 import _native, host, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def host_inputs(m: int, seed: int, pin: bool = True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((m, 6, 256), dtype=torch.bfloat16, generator=g)
    k = torch.randn((m, 1, 256), dtype=torch.bfloat16, generator=g)
    pos = torch.randint(0, 4096, (m,), generator=g, dtype=torch.int64)
    cache = workloads.make_cos_sin_cache(4096, 10000.0)
    if pin:
        q, k, pos = q.pin_memory(), k.pin_memory(), pos.pin_memory()
    return q, k, pos, cache


@pytest.mark.parametrize("m,chunk", [(1, 2048), (100, 2048), (2048, 2048), (5000, 2048), (777, 64), (9000, 1000)])
def test_host_entry_matches_oracle(m, chunk):
    q, k, pos, cache = host_inputs(m, m)
    q0, k0 = q.clone(), k.clone()
    host.welmv4_inplace_rope_host(q, k, pos, cache.to(DEV), chunk_tokens=chunk)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(q0, k0, pos, None, cache)
    assert torch.equal(q.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(k.view(torch.int16), k_ref.view(torch.int16))


def test_host_entry_repeated_calls_and_pageable_memory():
    q, k, pos, cache = host_inputs(3000, 1, pin=False)
    q0, k0 = q.clone(), k.clone()
    dcache = cache.to(DEV)
    for _ in range(3):
        host.welmv4_inplace_rope_host(q, k, pos, dcache, chunk_tokens=512)
    torch.cuda.synchronize()
    for _ in range(3):
        q0, k0 = rope_oracle.reference_outputs(q0, k0, pos, None, cache)
    assert torch.equal(q.view(torch.int16), q0.view(torch.int16))
    assert torch.equal(k.view(torch.int16), k0.view(torch.int16))


def test_host_entry_strided_host_views_and_device_positions():
    m = 1500
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn((m, 8 * 256), dtype=torch.bfloat16, generator=g).pin_memory()
    q = qkv[:, : 6 * 256].view(m, 6, 256)
    k = qkv[:, 6 * 256: 7 * 256].view(m, 1, 256)
    pos = torch.randint(0, 4096, (m,), generator=g, dtype=torch.int64)
    cache = workloads.make_cos_sin_cache(4096, 10000.0)
    before = qkv.clone()
    host.welmv4_inplace_rope_host(q, k, pos.to(DEV), cache.to(DEV), chunk_tokens=700)
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(before[:, :1536].reshape(m, 6, 256),
                                                 before[:, 1536:1792].reshape(m, 1, 256), pos, None, cache)
    assert torch.equal(q.reshape(m, 6, 256).view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(k.reshape(m, 1, 256).view(torch.int16), k_ref.view(torch.int16))
    assert torch.equal(qkv[:, 1792:], before[:, 1792:])  # the V head is never touched


def test_copy_rope_lanes_moves_only_rotated_lanes():
    m = 300
    src = torch.randn((m, 6, 256), dtype=torch.bfloat16).pin_memory()
    dst = torch.zeros((m, 6, 256), dtype=torch.bfloat16, device=DEV)
    stream = torch.cuda.current_stream()
    lib = _native.load()
    rc = lib.welm_rope_copy_rope_lanes(dst.data_ptr(), src.data_ptr(), m, 6, 1536, 1536, 0, stream.cuda_stream)
    assert rc == 0
    back = torch.full((m, 6, 256), 7.0, dtype=torch.bfloat16).pin_memory()
    rc = lib.welm_rope_copy_rope_lanes(back.data_ptr(), dst.data_ptr(), m, 6, 1536, 1536, 1, stream.cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(dst[..., 192:].cpu(), src[..., 192:])
    assert torch.count_nonzero(dst[..., :192]).item() == 0
    assert torch.equal(back[..., 192:], src[..., 192:])
    assert bool((back[..., :192] == 7.0).all())
