"""Reference-facing Python API of the B200 in-place partial RoPE.

The functions here mirror the reference's call surface for this op
(bench_welmv4_inplace_rope_npu.py):

* :func:`welmv4_inplace_rope_npu` — the production entry
  ``(q, k, positions, cos_sin_cache, last_index | None)`` of the frozen kernel
  (bench_welmv4_inplace_rope_npu.py:326-405): ordinary prefill / decode when
  ``last_index`` is None, KV-mirror prefill otherwise.
* :func:`rope_prefill` — the ordinary tiled kernel's runtime arguments
  ``(q, k, positions, cache, segment_tile_starts_or_placeholder,
  num_work_tiles, N, q_token_stride, k_token_stride, has_segments)``
  (bench_welmv4_inplace_rope_npu.py:679-690).
* :func:`rope_mirror_prefill` — the mirror kernel's runtime arguments
  ``(..., last_index, segment_tile_starts_or_placeholder, num_work_tiles, N,
  BS, q_token_stride, k_token_stride, has_segments)``
  (bench_welmv4_inplace_rope_npu.py:818-831).
* :func:`build_segment_tile_starts` — the segmented 64-token tile builder
  (bench_welmv4_inplace_rope_npu.py:1439-1461) and segmented ``last_index``
  (bench_welmv4_inplace_rope_npu.py:1402-1424), on the host or the device.

Every call goes to the sm_100a library through its C ABI on the current
CUDA stream; Q and K are rotated in place and nothing is returned.  Misuse
raises ``ValueError``/``TypeError`` on the host (as the reference's
``Harness.bind`` does, bench_welmv4_inplace_rope_npu.py:1177-1180,1208-1213,
1268-1271); a non-zero library status raises :class:`WelmRopeError`.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np
import torch

from . import _native
from ._native import WelmRopeError

HEAD_DIM = 256
ROPE_DIM = 64
NUM_Q_HEADS = 6
NUM_K_HEADS = 1
TILE_TOKENS = 64

__all__ = [
    "WelmRopeError",
    "welmv4_inplace_rope_npu",
    "welmv4_inplace_rope",
    "rope_prefill",
    "rope_mirror_prefill",
    "rope_mirror_from_lens",
    "rope_mirror_kv_write",
    "build_segment_tile_starts",
    "build_segment_tile_starts_device",
    "count_segment_tiles",
    "segment_placeholder",
]


# ---------------------------------------------------------------------------
# Argument checks (host only; never reads device memory).
# ---------------------------------------------------------------------------
def _require(t: Optional[torch.Tensor], name: str, dtype: torch.dtype, device: torch.device) -> None:
    if t is None:
        raise ValueError(f"{name} is required")
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _check_heads(t: torch.Tensor, name: str, heads: int) -> None:
    if t.dim() != 3 or tuple(t.shape[1:]) != (heads, HEAD_DIM):
        raise ValueError(f"{name} must have shape [rows, {heads}, {HEAD_DIM}], got {tuple(t.shape)}")
    if t.shape[0] > 0 and (t.stride(2) != 1 or (heads > 1 and t.stride(1) != HEAD_DIM)):
        raise ValueError(f"{name} heads must be contiguous (lane stride 1, head stride {HEAD_DIM})")


def _check_common(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor) -> torch.device:
    if not isinstance(q, torch.Tensor) or q.device.type != "cuda":
        raise ValueError("query must be a CUDA tensor (the op runs only on the sm_100a library)")
    device = q.device
    _require(q, "query", torch.bfloat16, device)
    _require(k, "key", torch.bfloat16, device)
    _require(positions, "positions", torch.int64, device)
    _require(cache, "cos_sin_cache", torch.float32, device)
    _check_heads(q, "query", NUM_Q_HEADS)
    _check_heads(k, "key", NUM_K_HEADS)
    if positions.dim() != 1 or (positions.numel() > 1 and positions.stride(0) != 1):
        raise ValueError("positions must be a contiguous 1-D int64 tensor")
    if cache.dim() != 2 or cache.shape[1] != ROPE_DIM or (cache.numel() and not cache.is_contiguous()):
        raise ValueError(f"cos_sin_cache must be a contiguous [max_position, {ROPE_DIM}] float32 tensor")
    return device


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else (t.data_ptr() or None)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _call(device: torch.device, fn, *args) -> int:
    """Run a library entry with ``device`` current: the library launches into
    the current device's context, and the tensors' device need not be the
    caller's current one."""
    if device.index is None or device.index == torch.cuda.current_device():
        return fn(*args)
    with torch.cuda.device(device):
        return fn(*args)


def _status_ptr(status: Optional[torch.Tensor], device: torch.device) -> Optional[int]:
    if status is None:
        return None
    _require(status, "status", torch.int32, device)
    if status.numel() < 1:
        raise ValueError("status must hold at least one int32")
    return status.data_ptr()


def _tiles(segment_tile_starts: Optional[torch.Tensor], has_segments: int, device: torch.device) -> Optional[int]:
    if has_segments not in (0, 1):
        raise ValueError(f"has_segments must be 0 or 1, got {has_segments}")
    if has_segments == 0:
        return None  # never dereferenced (a placeholder may be passed)
    _require(segment_tile_starts, "segment_tile_starts", torch.int32, device)
    if segment_tile_starts.dim() != 1 or (segment_tile_starts.numel() > 1 and segment_tile_starts.stride(0) != 1):
        raise ValueError("segment_tile_starts must be a contiguous 1-D int32 tensor")
    return segment_tile_starts.data_ptr()


# ---------------------------------------------------------------------------
# Reference launch surfaces.
# ---------------------------------------------------------------------------
def rope_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    segment_tile_starts: Optional[torch.Tensor],
    num_work_tiles: int,
    N: int,
    q_token_stride: int,
    k_token_stride: int,
    has_segments: int,
    status: Optional[torch.Tensor] = None,
) -> None:
    """Ordinary prefill / decode, with the ordinary tiled kernel's arguments.

    has_segments=0: tiles ``[64 i, min(64 i + 64, N))`` for ``i <
    num_work_tiles`` (pass ``ceil(N / 64)``); has_segments=1: tiles from
    ``segment_tile_starts`` (``num_work_tiles + 1`` entries).
    """
    device = _check_common(q, k, positions, cos_sin_cache)
    starts = _tiles(segment_tile_starts, int(has_segments), device)
    if has_segments and segment_tile_starts.numel() < int(num_work_tiles) + 1:
        raise ValueError("segment_tile_starts must hold num_work_tiles + 1 entries")
    if int(N) > positions.numel() or int(N) > k.shape[0] or int(N) > q.shape[0]:
        raise ValueError("N exceeds the rows of positions, key or query")
    lib = _native.load()
    rc = _call(device, lib.welm_rope_ordinary,
        _ptr(q), _ptr(k), _ptr(positions), _ptr(cos_sin_cache), starts,
        int(num_work_tiles), int(N), int(q_token_stride), int(k_token_stride),
        int(has_segments), int(cos_sin_cache.shape[0]), _status_ptr(status, device), _stream(device),
    )
    _native.check("welm_rope_ordinary", rc)


def rope_mirror_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    last_index: torch.Tensor,
    segment_tile_starts: Optional[torch.Tensor],
    num_work_tiles: int,
    N: int,
    BS: int,
    q_token_stride: int,
    k_token_stride: int,
    has_segments: int,
    status: Optional[torch.Tensor] = None,
) -> None:
    """KV-mirror prefill, with the mirror kernel's arguments.

    Q row ``b < BS`` is rotated at ``positions[last_index[b]]``; K rows follow
    the same tile rules as :func:`rope_prefill`.
    """
    device = _check_common(q, k, positions, cos_sin_cache)
    _require(last_index, "last_index", torch.int64, device)
    if last_index.dim() != 1 or (last_index.numel() > 1 and last_index.stride(0) != 1):
        raise ValueError("last_index must be a contiguous 1-D int64 tensor")
    starts = _tiles(segment_tile_starts, int(has_segments), device)
    if has_segments and segment_tile_starts.numel() < int(num_work_tiles) + 1:
        raise ValueError("segment_tile_starts must hold num_work_tiles + 1 entries")
    if int(BS) > q.shape[0] or int(BS) > last_index.numel():
        raise ValueError("BS exceeds the rows of query or last_index")
    if int(N) > positions.numel() or int(N) > k.shape[0]:
        raise ValueError("N exceeds the rows of positions or key")
    lib = _native.load()
    rc = _call(device, lib.welm_rope_mirror,
        _ptr(q), _ptr(k), _ptr(positions), _ptr(cos_sin_cache), _ptr(last_index), starts,
        int(num_work_tiles), int(N), int(BS), int(q_token_stride), int(k_token_stride),
        int(has_segments), int(cos_sin_cache.shape[0]), _status_ptr(status, device), _stream(device),
    )
    _native.check("welm_rope_mirror", rc)


def welmv4_inplace_rope_npu(
    query: torch.Tensor,
    key: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    last_index: Optional[torch.Tensor] = None,
    segment_tile_starts: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
) -> None:
    """Production entry: in-place tail RoPE on Q and K.

    ``last_index is None`` selects ordinary prefill / decode (Q has one row
    per token); otherwise KV-mirror prefill (Q has ``BS = last_index.numel()``
    rows, row b at ``positions[last_index[b]]``).  ``segment_tile_starts``
    (optional, int32 ``[T+1]``) selects the segmented tile source.
    """
    n_tokens = int(positions.shape[0]) if isinstance(positions, torch.Tensor) else 0
    has_segments = 0 if segment_tile_starts is None else 1
    tiles = (n_tokens + TILE_TOKENS - 1) // TILE_TOKENS if not has_segments else int(segment_tile_starts.numel()) - 1
    if last_index is None:
        if query.shape[0] != n_tokens or key.shape[0] != n_tokens:
            raise ValueError("ordinary RoPE needs query, key and positions with the same row count")
        rope_prefill(query, key, positions, cos_sin_cache, segment_tile_starts, tiles, n_tokens,
                     query.stride(0), key.stride(0), has_segments, status)
    else:
        batch = int(last_index.numel())
        if query.shape[0] != batch or key.shape[0] != n_tokens:
            raise ValueError("KV-mirror RoPE needs query rows == last_index.numel() and key rows == positions rows")
        rope_mirror_prefill(query, key, positions, cos_sin_cache, last_index, segment_tile_starts, tiles,
                            n_tokens, batch, query.stride(0), key.stride(0), has_segments, status)


welmv4_inplace_rope = welmv4_inplace_rope_npu


def rope_mirror_kv_write(
    q: torch.Tensor,
    q_out: torch.Tensor,
    k: torch.Tensor,
    v: Optional[torch.Tensor],
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    last_index: torch.Tensor,
    slot_mapping: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
) -> None:
    """KV-mirror prefill fused with the paged KV-cache write and the Q
    last-row extraction (one pass, inputs read only):

    * ``q_out[b] = rope(q[last_index[b]])`` — q is the full ``[N, 6, 256]``
      projection output, q_out has one row per request;
    * ``key_cache[slot] = rope(k[t])`` and ``value_cache[slot] = v[t]`` for
      ``slot = slot_mapping[t] >= 0`` (negative slots are padding tokens).

    Caches are contiguous bf16 tensors with one KV head of 256 lanes per slot,
    e.g. ``[num_blocks, block_size, 1, 256]`` or ``[num_blocks, 1,
    block_size, 256]`` (slot = block * block_size + offset in both).
    """
    device = _check_common(q, k, positions, cos_sin_cache)
    _require(q_out, "q_out", torch.bfloat16, device)
    _check_heads(q_out, "q_out", NUM_Q_HEADS)
    _require(last_index, "last_index", torch.int64, device)
    _require(slot_mapping, "slot_mapping", torch.int64, device)
    _require(key_cache, "key_cache", torch.bfloat16, device)
    if (v is None) != (value_cache is None):
        raise ValueError("pass both v and value_cache, or neither")
    if v is not None:
        _require(v, "v", torch.bfloat16, device)
        _check_heads(v, "v", NUM_K_HEADS)
        _require(value_cache, "value_cache", torch.bfloat16, device)
    for name, t in (("key_cache", key_cache), ("value_cache", value_cache)):
        if t is not None and (not t.is_contiguous() or t.numel() % HEAD_DIM):
            raise ValueError(f"{name} must be contiguous with {HEAD_DIM} lanes per slot")
    if value_cache is not None and value_cache.numel() != key_cache.numel():
        raise ValueError("key_cache and value_cache must hold the same number of slots")
    for name, t in (("last_index", last_index), ("slot_mapping", slot_mapping)):
        if t.dim() != 1 or (t.numel() > 1 and t.stride(0) != 1):
            raise ValueError(f"{name} must be a contiguous 1-D int64 tensor")
    n = int(positions.shape[0])
    batch = int(last_index.numel())
    if k.shape[0] != n or q.shape[0] < n or slot_mapping.numel() != n or (v is not None and v.shape[0] != n):
        raise ValueError("q, k, v and slot_mapping need one row per token")
    if q_out.shape[0] != batch:
        raise ValueError("q_out needs one row per request (last_index entry)")
    rc = _call(device, _native.load().welm_rope_mirror_kv_write,
        _ptr(q), _ptr(q_out), _ptr(k), _ptr(v), _ptr(positions), _ptr(cos_sin_cache), _ptr(last_index),
        _ptr(slot_mapping), _ptr(key_cache), _ptr(value_cache), n, batch, int(q.stride(0)), int(q_out.stride(0)),
        int(k.stride(0)), int(v.stride(0)) if v is not None else 0, HEAD_DIM, key_cache.numel() // HEAD_DIM,
        int(cos_sin_cache.shape[0]), _status_ptr(status, device), _stream(device))
    _native.check("welm_rope_mirror_kv_write", rc)


def rope_mirror_from_lens(
    q: torch.Tensor,
    k: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    seq_lens: torch.Tensor,
    status: Optional[torch.Tensor] = None,
) -> None:
    """Segmented KV-mirror prefill from device request lengths (no tile table,
    no last_index, no host round trip): K token t < sum(seq_lens) at
    positions[t]; Q row r at positions[seq_lens[0] + ... + seq_lens[r] - 1].
    Equals build_segment_tile_starts_device + rope_mirror_prefill."""
    device = _check_common(q, k, positions, cos_sin_cache)
    _require(seq_lens, "seq_lens", torch.int64, device)
    if seq_lens.dim() != 1 or (seq_lens.numel() > 1 and seq_lens.stride(0) != 1):
        raise ValueError("seq_lens must be a contiguous 1-D int64 tensor")
    batch = int(seq_lens.numel())
    if batch > _native.LENS_MAX_BATCH:
        raise ValueError(f"at most {_native.LENS_MAX_BATCH} requests per call")
    if q.shape[0] != batch:
        raise ValueError("query needs one row per request")
    n = int(positions.shape[0])
    if k.shape[0] != n:
        raise ValueError("key rows must equal the positions length")
    rc = _call(device, _native.load().welm_rope_mirror_from_lens,
        _ptr(q), _ptr(k), _ptr(positions), _ptr(cos_sin_cache), _ptr(seq_lens), n, batch, int(q.stride(0)),
        int(k.stride(0)), int(cos_sin_cache.shape[0]), _status_ptr(status, device), _stream(device))
    _native.check("welm_rope_mirror_from_lens", rc)


# ---------------------------------------------------------------------------
# Segmented tile builder.
# ---------------------------------------------------------------------------
def _lens_array(seq_lens: Sequence[int] | np.ndarray | torch.Tensor) -> np.ndarray:
    if isinstance(seq_lens, torch.Tensor):
        seq_lens = seq_lens.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(seq_lens, dtype=np.int64).reshape(-1))


def count_segment_tiles(seq_lens: Sequence[int] | np.ndarray | torch.Tensor) -> int:
    """T = sum ceil(len / 64) (host twin, C ABI)."""
    lens = _lens_array(seq_lens)
    out = ctypes.c_int64(0)
    rc = _native.load().welm_rope_count_tiles_host(lens.ctypes.data if lens.size else None, lens.size, ctypes.byref(out))
    _native.check("welm_rope_count_tiles_host", rc)
    return int(out.value)


def build_segment_tile_starts(
    seq_lens: Sequence[int] | np.ndarray | torch.Tensor,
    device: torch.device | str | None = None,
) -> tuple[torch.Tensor, int, torch.Tensor]:
    """Host builder: returns (tile_starts int32 [T+1], T, last_index int64 [BS]).

    The tables are built on the host by the C twin and, when ``device`` is
    given, copied there once (as the reference builds them "once before the
    launch").
    """
    lens = _lens_array(seq_lens)
    tiles = count_segment_tiles(lens)
    starts = np.empty(tiles + 1, dtype=np.int32)
    last = np.empty(lens.size, dtype=np.int64)
    out_t = ctypes.c_int64(0)
    rc = _native.load().welm_rope_build_tiles_host(
        lens.ctypes.data if lens.size else None, lens.size, starts.ctypes.data, starts.size,
        ctypes.byref(out_t), last.ctypes.data if last.size else None,
    )
    _native.check("welm_rope_build_tiles_host", rc)
    starts_t = torch.from_numpy(starts)
    last_t = torch.from_numpy(last)
    if device is not None:
        starts_t = starts_t.to(device)
        last_t = last_t.to(device)
    return starts_t, int(out_t.value), last_t


def build_segment_tile_starts_device(
    seq_lens: torch.Tensor,
    capacity: Optional[int] = None,
    status: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Device builder: returns (tile_starts int32 [capacity], num_tiles int32 [1],
    last_index int64 [BS]), all on ``seq_lens.device``; nothing is synchronised.

    The host does not know the lengths, so ``capacity`` (int32 slots for the
    starts) is required when ``BS > 0``; ``ceil(N / 64) + BS + 1`` always
    suffices for ``N`` total tokens.  The tile count stays on the device in
    ``num_tiles``; reading it on the host is the caller's synchronisation.
    """
    if not isinstance(seq_lens, torch.Tensor) or seq_lens.device.type != "cuda":
        raise ValueError("seq_lens must be a CUDA int64 tensor")
    device = seq_lens.device
    _require(seq_lens, "seq_lens", torch.int64, device)
    lens = seq_lens.contiguous()
    batch = int(lens.numel())
    if capacity is None:
        if batch:
            raise ValueError("capacity is required (ceil(N/64) + BS + 1 always suffices)")
        capacity = 1
    starts = torch.empty(int(capacity), dtype=torch.int32, device=device)
    num_tiles = torch.empty(1, dtype=torch.int32, device=device)
    last = torch.empty(batch, dtype=torch.int64, device=device)
    rc = _call(device, _native.load().welm_rope_build_tiles,
        _ptr(lens), batch, starts.data_ptr(), int(capacity), num_tiles.data_ptr(), _ptr(last),
        _status_ptr(status, device), _stream(device),
    )
    _native.check("welm_rope_build_tiles", rc)
    return starts, num_tiles, last


def segment_placeholder(device: torch.device | str) -> torch.Tensor:
    """Stable int32[2] placeholder for non-segmented launches
    (bench_welmv4_inplace_rope_npu.py:1136-1140); never dereferenced."""
    return torch.zeros((2,), dtype=torch.int32, device=device)


# ---------------------------------------------------------------------------
# torch.library registration: `torch.ops.welm_b200.inplace_rope`.
# ---------------------------------------------------------------------------
@torch.library.custom_op("welm_b200::inplace_rope", mutates_args=("query", "key"))
def _inplace_rope_op(
    query: torch.Tensor,
    key: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    last_index: Optional[torch.Tensor] = None,
    segment_tile_starts: Optional[torch.Tensor] = None,
) -> None:
    welmv4_inplace_rope_npu(query, key, positions, cos_sin_cache, last_index, segment_tile_starts)


@_inplace_rope_op.register_fake
def _inplace_rope_fake(query, key, positions, cos_sin_cache, last_index=None, segment_tile_starts=None) -> None:
    return None
