"""GPU tests of the host-memory entry (welmv4_inplace_rope_host) over both
transports (the mapped kernel on pinned memory and the staged copy
pipeline), the mapped C-ABI entry and the rope-lane copy helper: results
must equal the oracle bit for bit and lanes 0..191 of the host tensors must
stay untouched."""

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


@pytest.mark.parametrize("transport", ["mapped", "staged"])
@pytest.mark.parametrize("m,chunk", [(1, 2048), (100, 2048), (2048, 2048), (5000, 2048), (777, 64), (9000, 1000),
                                     (16384, 2048), (40000, 4096)])  # 40000: the mapped grid strides twice
def test_host_entry_matches_oracle(m, chunk, transport):
    q, k, pos, cache = host_inputs(m, m)
    q0, k0 = q.clone(), k.clone()
    host.welmv4_inplace_rope_host(q, k, pos, cache.to(DEV), chunk_tokens=chunk, transport=transport)
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


@pytest.mark.parametrize("transport", ["mapped", "staged"])
def test_host_entry_strided_host_views_and_device_positions(transport):
    m = 1500
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn((m, 8 * 256), dtype=torch.bfloat16, generator=g).pin_memory()
    q = qkv[:, : 6 * 256].view(m, 6, 256)
    k = qkv[:, 6 * 256: 7 * 256].view(m, 1, 256)
    pos = torch.randint(0, 4096, (m,), generator=g, dtype=torch.int64)
    cache = workloads.make_cos_sin_cache(4096, 10000.0)
    before = qkv.clone()
    host.welmv4_inplace_rope_host(q, k, pos.to(DEV), cache.to(DEV), chunk_tokens=700, transport=transport)
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


def mapped_call(q, k, pos, cache, status=None, n=None):
    stream = torch.cuda.current_stream()
    return _native.load().welm_rope_ordinary_mapped(
        q.data_ptr(), k.data_ptr(), pos.data_ptr(), cache.data_ptr(), q.shape[0] if n is None else n,
        q.stride(0), k.stride(0), cache.shape[0], None if status is None else status.data_ptr(),
        stream.cuda_stream)


def test_mapped_entry_skips_out_of_range_positions_and_reports_them():
    q, k, pos, cache = host_inputs(333, 9)
    pos[5], pos[200], pos[332] = -1, 4096, 1 << 40
    q0, k0 = q.clone(), k.clone()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dcache = cache.to(DEV)
    assert mapped_call(q, k, pos, dcache, status) == 0
    torch.cuda.synchronize()
    assert status.item() == _native.DEV_BAD_POSITION
    good = torch.ones(333, dtype=torch.bool)
    good[[5, 200, 332]] = False
    q_ref, k_ref = rope_oracle.reference_outputs(q0[good], k0[good], pos[good], None, cache)
    assert torch.equal(q[good].view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(k[good].view(torch.int16), k_ref.view(torch.int16))
    assert torch.equal(q[~good].view(torch.int16), q0[~good].view(torch.int16))
    assert torch.equal(k[~good].view(torch.int16), k0[~good].view(torch.int16))


def test_mapped_entry_rejects_memory_the_device_cannot_reach():
    q, k, pos, cache = host_inputs(64, 4)
    dcache = cache.to(DEV)
    pageable_q = q.clone()  # clone() of a pinned tensor is pageable
    assert not pageable_q.is_pinned()
    before = pageable_q.clone()
    assert mapped_call(pageable_q, k, pos, dcache) == _native.ERR_NOT_MAPPED
    assert mapped_call(q, k, pos.clone(), dcache) == _native.ERR_NOT_MAPPED  # pageable positions
    dev_q = q.to(DEV)  # device Q is not host memory
    assert mapped_call(dev_q, k, pos, dcache) == _native.ERR_NOT_MAPPED
    torch.cuda.synchronize()
    assert torch.equal(pageable_q, before)
    with pytest.raises(Exception, match="not page-locked"):
        host.welmv4_inplace_rope_host(pageable_q, k, pos, dcache, transport="mapped")


def test_misaligned_pinned_views_take_the_staged_transport():
    m = 200
    g = torch.Generator().manual_seed(5)
    buf = torch.randn((m * 1536 + 8,), dtype=torch.bfloat16, generator=g).pin_memory()
    q = buf[1: 1 + m * 1536].view(m, 6, 256)  # 2-byte offset: not 16-byte aligned
    k = torch.randn((m, 1, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    pos = torch.randint(0, 4096, (m,), generator=g, dtype=torch.int64)
    cache = workloads.make_cos_sin_cache(4096, 10000.0)
    dcache = cache.to(DEV)
    assert mapped_call(q, k, pos.pin_memory(), dcache) == _native.ERR_BAD_STRIDE
    q0, k0 = q.clone(), k.clone()
    host.welmv4_inplace_rope_host(q, k, pos, dcache)  # auto: staged
    torch.cuda.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(q0, k0, pos, None, cache)
    assert torch.equal(q.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(k.view(torch.int16), k_ref.view(torch.int16))


def test_mapped_entry_on_a_side_stream_after_device_work():
    q, k, pos, cache = host_inputs(4096, 11)
    q0, k0 = q.clone(), k.clone()
    dcache = cache.to(DEV)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        dpos = pos.to(DEV, non_blocking=True)
        host.welmv4_inplace_rope_host(q, k, dpos, dcache, transport="mapped")
    side.synchronize()
    q_ref, k_ref = rope_oracle.reference_outputs(q0, k0, pos, None, cache)
    assert torch.equal(q.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(k.view(torch.int16), k_ref.view(torch.int16))
