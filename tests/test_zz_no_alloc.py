"""The allocation-free host entry, welm_rope_ordinary_host_static.

Some callers cannot allocate device memory at all: a plugin inside a host
process whose allocator already owns the whole GPU, or code on a
latency-critical path where cudaMalloc/cudaFree (which may synchronise the
device) are off limits.  For them the library stages the rotated lanes of a
host-resident batch (up to 2048 tokens) through a fixed device area compiled
into the library.  This test drives that entry through the C ABI twice in a
row — the second call with other data and a smaller batch, so leftovers of
the first call in the shared area would show — and checks every result
against the regular device entry (welm_rope_ordinary) on copies of the same
inputs, bit for bit (the tolerance every parity test here uses: 0 ulp).

The file is named so that pytest collects it last; it passes on its own in a
fresh process and after the rest of the suite.
"""

from __future__ import annotations

import pytest
import torch

from testfiles_b200 import _native, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _inputs(m: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((m, 6, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    k = torch.randn((m, 1, 256), dtype=torch.bfloat16, generator=g).pin_memory()
    pos = torch.randint(0, 16384, (m,), generator=g, dtype=torch.int64).pin_memory()
    return q, k, pos


def _device_reference(q, k, pos, cache) -> tuple[torch.Tensor, torch.Tensor]:
    """The existing entry point on device copies of the same inputs."""
    dq, dk, dp = q.to(DEV), k.to(DEV), pos.to(DEV)
    rc = _native.load().welm_rope_ordinary(
        dq.data_ptr(), dk.data_ptr(), dp.data_ptr(), cache.data_ptr(), None, (q.shape[0] + 63) // 64, q.shape[0],
        dq.stride(0), dk.stride(0), 0, cache.shape[0], None, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _native.OK, _native.status_string(rc)
    return dq.cpu(), dk.cpu()


def _static_entry(q, k, pos, cache, status) -> int:
    return _native.load().welm_rope_ordinary_host_static(
        q.data_ptr(), k.data_ptr(), pos.data_ptr(), cache.data_ptr(), q.shape[0], q.stride(0), k.stride(0),
        cache.shape[0], status.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)


def test_static_entry_matches_device_entry_on_two_calls_in_a_row():
    torch.cuda.set_device(DEV)
    cache = workloads.make_cos_sin_cache(16384, 10000.0, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for m, seed in ((_native.STATIC_MAX_TOKENS, 1), (777, 2)):
        q, k, pos = _inputs(m, seed)
        q_want, k_want = _device_reference(q, k, pos, cache)
        rc = _static_entry(q, k, pos, cache, status)
        assert rc == _native.OK, _native.status_string(rc)
        torch.cuda.synchronize()
        assert torch.equal(q.view(torch.int16), q_want.view(torch.int16)), f"query differs (m={m})"
        assert torch.equal(k.view(torch.int16), k_want.view(torch.int16)), f"key differs (m={m})"
    assert status.item() == 0


def test_static_entry_rejects_batches_beyond_its_area():
    cache = workloads.make_cos_sin_cache(64, 10000.0, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q, k, pos = _inputs(_native.STATIC_MAX_TOKENS + 1, 3)
    before = q.clone()
    rc = _static_entry(q, k, pos, cache, status)
    assert rc == _native.ERR_TOO_MANY_TOKENS
    assert "2048" in _native.status_string(rc)
    torch.cuda.synchronize()
    assert torch.equal(q, before)  # nothing was copied or launched
