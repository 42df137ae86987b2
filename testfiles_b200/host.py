"""In-place RoPE on Q/K that live in host memory.

``welmv4_inplace_rope_host(query, key, positions, cos_sin_cache)`` rotates
host-resident Q ``[M, 6, 256]`` and K ``[M, 1, 256]`` (ordinary prefill /
decode) in place with the B200 kernels.  Only the rotated lanes (192..255)
cross PCIe — the op reads and writes nothing else.  Two transports:

* ``"mapped"`` (the default for pinned Q/K): one kernel
  (``welm_rope_ordinary_mapped``) reads every 128-byte rope slice straight
  from the pinned host tensors, rotates it and writes it back, so reads and
  writes share the bus in both directions at once.  No staging, no copies.
* ``"staged"`` (pageable Q/K, or on request): the batch is split into chunks
  that flow through a three-stage pipeline on separate CUDA streams —
  ``welm_rope_copy_rope_lanes`` in, the device kernel, copy back — with three
  device staging slots allocated once per device and chunk size by this
  Python layer.

Either way the call is stream-ordered like a device op: it starts after the
work already queued on the current stream, and the host tensors hold the
result once the current stream is synchronised.  The C ABI underneath never
allocates.
"""

from __future__ import annotations

import threading
from typing import Optional

import torch

from . import _native, ops

HEAD_DIM = ops.HEAD_DIM
NUM_Q_HEADS = ops.NUM_Q_HEADS
DEFAULT_CHUNK_TOKENS = 2048
SLOTS = 3

_pipelines: dict[tuple[int, int], "HostRopePipeline"] = {}
_lock = threading.Lock()


def _copy_lanes(dst: torch.Tensor, src: torch.Tensor, rows: int, heads: int, direction: int, stream) -> None:
    rc = _native.load().welm_rope_copy_rope_lanes(
        dst.data_ptr(), src.data_ptr(), rows, heads, dst.stride(0), src.stride(0), direction, stream.cuda_stream)
    _native.check("welm_rope_copy_rope_lanes", rc)


class HostRopePipeline:
    """Staging buffers, streams and events for one device and chunk size."""

    def __init__(self, device: torch.device, chunk_tokens: int = DEFAULT_CHUNK_TOKENS):
        if chunk_tokens <= 0:
            raise ValueError("chunk_tokens must be positive")
        self.device = device
        self.chunk = int(chunk_tokens)
        self.q = [torch.empty((self.chunk, NUM_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
                  for _ in range(SLOTS)]
        self.k = [torch.empty((self.chunk, 1, HEAD_DIM), dtype=torch.bfloat16, device=device)
                  for _ in range(SLOTS)]
        self.p = [torch.empty(self.chunk, dtype=torch.int64, device=device) for _ in range(SLOTS)]
        self.h2d = torch.cuda.Stream(device)
        self.compute = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.loaded = [torch.cuda.Event() for _ in range(SLOTS)]
        self.rotated = [torch.cuda.Event() for _ in range(SLOTS)]
        self.freed = [torch.cuda.Event() for _ in range(SLOTS)]
        self.used = [False] * SLOTS
        self.lock = threading.Lock()

    def run(self, query: torch.Tensor, key: torch.Tensor, positions: torch.Tensor,
            cos_sin_cache: torch.Tensor) -> None:
        n = int(positions.shape[0])
        if n == 0:
            return
        current = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device), self.lock:  # the pipeline's device, whatever is current
            self.h2d.wait_stream(current)
            for c, t0 in enumerate(range(0, n, self.chunk)):
                t1 = min(n, t0 + self.chunk)
                rows = t1 - t0
                s = c % SLOTS
                dq, dk, dp = self.q[s], self.k[s], self.p[s]
                if self.used[s]:
                    self.h2d.wait_event(self.freed[s])
                with torch.cuda.stream(self.h2d):
                    _copy_lanes(dq, query[t0:t1], rows, NUM_Q_HEADS, 0, self.h2d)
                    _copy_lanes(dk, key[t0:t1], rows, 1, 0, self.h2d)
                    dp[:rows].copy_(positions[t0:t1], non_blocking=True)
                    self.loaded[s].record(self.h2d)
                self.compute.wait_event(self.loaded[s])
                with torch.cuda.stream(self.compute):
                    ops.rope_prefill(dq, dk, dp, cos_sin_cache, None, (rows + 63) // 64, rows,
                                     dq.stride(0), dk.stride(0), 0)
                    self.rotated[s].record(self.compute)
                self.d2h.wait_event(self.rotated[s])
                with torch.cuda.stream(self.d2h):
                    _copy_lanes(query[t0:t1], dq, rows, NUM_Q_HEADS, 1, self.d2h)
                    _copy_lanes(key[t0:t1], dk, rows, 1, 1, self.d2h)
                    self.freed[s].record(self.d2h)
                self.used[s] = True
            current.wait_stream(self.d2h)


def _check_host(t: torch.Tensor, name: str, dtype: torch.dtype, heads: Optional[int] = None) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
        raise ValueError(f"{name} must be a host (CPU) tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if heads is not None:
        if t.dim() != 3 or tuple(t.shape[1:]) != (heads, HEAD_DIM):
            raise ValueError(f"{name} must have shape [rows, {heads}, {HEAD_DIM}]")
        if t.shape[0] and (t.stride(2) != 1 or t.stride(1) != HEAD_DIM or t.stride(0) < heads * HEAD_DIM):
            raise ValueError(f"{name} must have contiguous heads and non-overlapping rows")


def _mapped(query: torch.Tensor, key: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor,
            device: torch.device) -> None:
    if positions.device.type == "cpu" and not (positions.is_pinned() and positions.is_contiguous()):
        positions = positions.contiguous().to(device)  # the kernel reads pinned or device positions only
    elif positions.device.type == "cuda":
        positions = positions.contiguous()
    stream = torch.cuda.current_stream(device)
    with torch.cuda.device(device):
        rc = _native.load().welm_rope_ordinary_mapped(
            query.data_ptr(), key.data_ptr(), positions.data_ptr(), cos_sin_cache.data_ptr(),
            int(positions.shape[0]), query.stride(0), key.stride(0), int(cos_sin_cache.shape[0]), None,
            stream.cuda_stream)
    _native.check("welm_rope_ordinary_mapped", rc)


def _mappable(t: torch.Tensor) -> bool:
    return (t.is_pinned() and t.data_ptr() % 16 == 0
            and (t.shape[0] <= 1 or t.stride(0) % 8 == 0))


def welmv4_inplace_rope_host(
    query: torch.Tensor,
    key: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    chunk_tokens: int = DEFAULT_CHUNK_TOKENS,
    transport: str = "auto",
) -> None:
    """Ordinary prefill / decode RoPE on host-resident Q/K (see module doc).

    ``positions`` may be on the host or the device; ``cos_sin_cache`` lives on
    the device that runs the op.  ``transport`` is ``"auto"`` (mapped when Q
    and K are pinned, 16-byte aligned with strides of 8 elements; staged
    otherwise), ``"mapped"`` or ``"staged"``.
    """
    if transport not in ("auto", "mapped", "staged"):
        raise ValueError("transport must be 'auto', 'mapped' or 'staged'")
    if not isinstance(cos_sin_cache, torch.Tensor) or cos_sin_cache.device.type != "cuda":
        raise ValueError("cos_sin_cache must be a CUDA tensor (it selects the device)")
    _check_host(query, "query", torch.bfloat16, NUM_Q_HEADS)
    _check_host(key, "key", torch.bfloat16, 1)
    if not isinstance(positions, torch.Tensor) or positions.dtype != torch.int64 or positions.dim() != 1:
        raise TypeError("positions must be a 1-D int64 tensor")
    n = int(positions.shape[0])
    if query.shape[0] != n or key.shape[0] != n:
        raise ValueError("query, key and positions need the same row count")
    device = cos_sin_cache.device
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if n == 0:
        return
    if transport == "mapped" or (transport == "auto" and _mappable(query) and _mappable(key)):
        _mapped(query, key, positions, cos_sin_cache, device)
        return
    key_ = (device.index, int(chunk_tokens))
    with _lock:
        pipe = _pipelines.get(key_)
        if pipe is None:
            pipe = _pipelines[key_] = HostRopePipeline(torch.device("cuda", key_[0]), chunk_tokens)
    pipe.run(query, key, positions, cos_sin_cache)


def lane_bytes(n_tokens: int) -> tuple[int, int]:
    """(host->device, device->host) bytes one call moves for n tokens."""
    slices = n_tokens * (NUM_Q_HEADS + 1) * 64 * 2
    return slices + n_tokens * 8, slices
