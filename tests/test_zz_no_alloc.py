"""The allocation-free host entry, welm_rope_ordinary_host_static.

Some callers cannot allocate device memory at all: a plugin inside a host
process whose allocator already owns the whole GPU, or code on a
latency-critical path where cudaMalloc/cudaFree (which may synchronise the
device) are off limits.  For them the library stages the rotated lanes of a
host-resident batch (up to 2048 tokens) through a fixed device area compiled
into the library.  These tests drive that entry through the C ABI:

* two calls in a row — the second with other data and a smaller batch, so
  leftovers of the first call in the shared area would show — each checked
  bit for bit (0 ulp, the tolerance every parity test here uses) against the
  oracle and against the regular device entry (welm_rope_ordinary) run on
  device copies of the same inputs;
* Q and K as strided views of a fused QKV buffer (token stride 2048), which
  take the per-head copy path instead of the single 2-D copy;
* an out-of-range position, which must set the status bit and leave that
  token exactly as it was.

The file is named so that pytest collects it last; it passes on its own in a
fresh process and after the rest of the suite.
"""

from __future__ import annotations

import pytest
import torch

from oracle import rope_oracle
from testfiles_b200 import _native, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAX_POSITION = 16384


def _packed(m: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((m, 6, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    k = torch.randn((m, 1, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    pos = torch.randint(0, MAX_POSITION, (m,), generator=g, dtype=torch.int64).pin_memory()
    return q, k, pos


def _fused_views(m: int, seed: int):
    """Q and K as views of one pinned [m, 8, 256] QKV buffer (token stride 2048)."""
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn((m, 8, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    pos = torch.randint(0, MAX_POSITION, (m,), generator=g, dtype=torch.int64).pin_memory()
    return qkv, qkv[:, :6], qkv[:, 6:7], pos


def _oracle(q, k, pos, cache_cpu) -> tuple[torch.Tensor, torch.Tensor]:
    return rope_oracle.reference_outputs(q.contiguous(), k.contiguous(), pos, None, cache_cpu)


def _device_entry(q, k, pos, cache) -> tuple[torch.Tensor, torch.Tensor]:
    """The existing entry point on device copies of the same inputs."""
    dq, dk, dp = q.contiguous().to(DEV), k.contiguous().to(DEV), pos.to(DEV)
    rc = _native.load().welm_rope_ordinary(
        dq.data_ptr(), dk.data_ptr(), dp.data_ptr(), cache.data_ptr(), None, (q.shape[0] + 63) // 64, q.shape[0],
        dq.stride(0), dk.stride(0), 0, cache.shape[0], None, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _native.OK, _native.status_string(rc)
    return dq.cpu(), dk.cpu()


def _static_entry(q, k, pos, cache, status) -> int:
    return _native.load().welm_rope_ordinary_host_static(
        q.data_ptr(), k.data_ptr(), pos.data_ptr(), cache.data_ptr(), q.shape[0], q.stride(0), k.stride(0),
        cache.shape[0], status.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


@pytest.fixture(scope="module")
def caches():
    torch.cuda.set_device(DEV)
    cpu = workloads.make_cos_sin_cache(MAX_POSITION, 10000.0)
    return cpu, cpu.to(DEV)


def test_static_entry_matches_oracle_and_device_entry_on_two_calls_in_a_row(caches):
    cache_cpu, cache = caches
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for m, seed in ((_native.STATIC_MAX_TOKENS, 1), (777, 2)):
        q, k, pos = _packed(m, seed)
        q_ref, k_ref = _oracle(q, k, pos, cache_cpu)
        q_dev, k_dev = _device_entry(q, k, pos, cache)
        rc = _static_entry(q, k, pos, cache, status)
        assert rc == _native.OK, _native.status_string(rc)
        torch.cuda.synchronize()
        assert _same_bits(q, q_ref) and _same_bits(k, k_ref), f"differs from the oracle (m={m})"
        assert _same_bits(q, q_dev) and _same_bits(k, k_dev), f"differs from welm_rope_ordinary (m={m})"
    assert status.item() == 0


def test_static_entry_on_fused_qkv_views(caches):
    """Token stride 2048: every head's lanes are copied with their own 2-D copy."""
    cache_cpu, cache = caches
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for m, seed in ((1500, 4), (33, 5)):
        qkv, q, k, pos = _fused_views(m, seed)
        assert q.stride(0) == 2048 and k.stride(0) == 2048
        v_before = qkv[:, 7].clone()
        q_ref, k_ref = _oracle(q, k, pos, cache_cpu)
        q_dev, k_dev = _device_entry(q, k, pos, cache)
        rc = _static_entry(q, k, pos, cache, status)
        assert rc == _native.OK, _native.status_string(rc)
        torch.cuda.synchronize()
        assert _same_bits(q, q_ref) and _same_bits(k, k_ref), f"differs from the oracle (m={m})"
        assert _same_bits(q, q_dev) and _same_bits(k, k_dev), f"differs from welm_rope_ordinary (m={m})"
        assert _same_bits(qkv[:, 7], v_before), "the V head beside Q and K was written"
    assert status.item() == 0


def test_static_entry_flags_an_out_of_range_position(caches):
    cache_cpu, cache = caches
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q, k, pos = _packed(300, 6)
    bad = 123
    pos[bad] = MAX_POSITION  # one past the cache's last row
    q_before, k_before = q.clone(), k.clone()
    good = torch.ones(300, dtype=torch.bool)
    good[bad] = False
    pos_ok = pos.clone()
    pos_ok[bad] = 0
    q_ref, k_ref = _oracle(q, k, pos_ok, cache_cpu)
    rc = _static_entry(q, k, pos, cache, status)
    assert rc == _native.OK, _native.status_string(rc)
    torch.cuda.synchronize()
    assert status.item() & _native.DEV_BAD_POSITION
    assert _same_bits(q[bad], q_before[bad]) and _same_bits(k[bad], k_before[bad]), "the flagged token changed"
    assert _same_bits(q[good], q_ref[good]) and _same_bits(k[good], k_ref[good]), "another token differs"


def test_static_entry_rejects_batches_beyond_its_area():
    cache = workloads.make_cos_sin_cache(64, 10000.0, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q, k, pos = _packed(_native.STATIC_MAX_TOKENS + 1, 3)
    before = q.clone()
    rc = _static_entry(q, k, pos, cache, status)
    assert rc == _native.ERR_TOO_MANY_TOKENS
    assert "2048" in _native.status_string(rc)
    torch.cuda.synchronize()
    assert torch.equal(q, before)  # nothing was copied or launched
