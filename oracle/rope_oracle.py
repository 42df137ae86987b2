"""CPU oracle for WeLMv4 in-place partial RoPE — TEST INFRASTRUCTURE ONLY.

This module checks the product and is never part of it: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference leg
may import it.  The product path (``testfiles_b200``) never calls it and has
no CPU fallback.

It restates, in plain torch-on-CPU and Python, the reference's algorithm for
this path (bench_welmv4_inplace_rope_npu.py):

* :func:`apply_reference`     — bench_welmv4_inplace_rope_npu.py:1489-1505
* :func:`reference_outputs`   — bench_welmv4_inplace_rope_npu.py:1508-1521
* :func:`make_cos_sin_cache`  — bench_welmv4_inplace_rope_npu.py:1391-1399
* :func:`make_last_index`     — bench_welmv4_inplace_rope_npu.py:1402-1424
* :func:`build_tile_starts`   — bench_welmv4_inplace_rope_npu.py:1439-1461
* :func:`make_uneven_segment_lens` — bench_welmv4_inplace_rope_npu.py:115-122

Arithmetic is the reference's: BF16 inputs widened to FP32, ``x1*c - x2*s``
and ``x1*s + x2*c`` as separate FP32 tensor ops (each product, the
difference and the sum rounded on its own), one cast to BF16
(round-to-nearest-even).  Lanes 0..191 are copied untouched.

Parity is pinned by ``tests/golden`` (outputs of the reference itself,
imported from its own source in the container that generated the fixtures;
see ``tests/golden/gen_golden.py``).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

HEAD_DIM = 256
ROPE_DIM = 64
HALF_ROPE_DIM = ROPE_DIM // 2
TILE_TOKENS = 64
DTYPE = torch.bfloat16


def apply_reference(data: torch.Tensor, rope_positions: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
    """Tail RoPE of every head of ``data`` [rows, heads, 256] at
    ``rope_positions`` [rows]; returns a new tensor."""
    output = data.clone()
    cos_sin = cache.index_select(0, rope_positions)
    cos = cos_sin[:, :HALF_ROPE_DIM].float().unsqueeze(1)
    sin = cos_sin[:, HALF_ROPE_DIM:].float().unsqueeze(1)
    rotary = data[..., HEAD_DIM - ROPE_DIM:]
    x1 = rotary[..., :HALF_ROPE_DIM].float()
    x2 = rotary[..., HALF_ROPE_DIM:].float()
    first = x1 * cos - x2 * sin
    second = x1 * sin + x2 * cos
    output[..., HEAD_DIM - ROPE_DIM:HEAD_DIM - HALF_ROPE_DIM] = first.to(DTYPE)
    output[..., HEAD_DIM - HALF_ROPE_DIM:] = second.to(DTYPE)
    return output


def reference_outputs(
    query: torch.Tensor,
    key: torch.Tensor,
    positions: torch.Tensor,
    last_index: Optional[torch.Tensor],
    cache: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(Q_out, K_out): Q rows at ``positions`` (ordinary) or at
    ``positions[last_index]`` (KV mirror); K rows at ``positions``."""
    query_positions = positions if last_index is None else positions.index_select(0, last_index)
    return apply_reference(query, query_positions, cache), apply_reference(key, positions, cache)


def make_cos_sin_cache(max_position: int, base: float, rope_dim: int = ROPE_DIM) -> torch.Tensor:
    """FP32 [max_position, rope_dim]: cos(p * f_i) then sin(p * f_i),
    f_i = 1 / base**(2i / rope_dim)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rope_dim, 2, dtype=torch.float32) / rope_dim))
    pos = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(torch.float32)


def build_tile_starts(segment_lens: Sequence[int]) -> list[int]:
    """Per-request 64-token tile starts followed by the total token count."""
    starts: list[int] = []
    token = 0
    for length in segment_lens:
        if length < 0:
            raise ValueError("negative request length")
        starts.extend(range(token, token + length, TILE_TOKENS))
        token += length
    starts.append(token)
    return starts


def make_last_index(n_tokens: int, batch_size: int, segment_lens: Sequence[int] = ()) -> list[int]:
    """Segmented: cumulative length minus one per request.  Otherwise the
    legacy evenly spaced rows ``(i + 1) * N // BS - 1`` clamped to [0, N-1]."""
    if segment_lens:
        out, end = [], 0
        for length in segment_lens:
            end += length
            out.append(end - 1)
        if end != n_tokens or len(out) != batch_size:
            raise ValueError("segmented mirror metadata is inconsistent")
        return out
    return [max(0, min(n_tokens - 1, (i + 1) * n_tokens // batch_size - 1)) for i in range(batch_size)]


def make_uneven_segment_lens(total: int, batch_size: int) -> tuple[int, ...]:
    """Positive, non-64-aligned lengths with an exact total: base +
    (-31, -17, -9, -1, 1, 9, 17, 31) cyclically, remainder on the last one."""
    pattern = (-31, -17, -9, -1, 1, 9, 17, 31)
    base = total // batch_size
    lengths = [base + pattern[i % len(pattern)] for i in range(batch_size)]
    lengths[-1] += total - sum(lengths)
    if min(lengths) <= 0 or sum(lengths) != total:
        raise ValueError("cannot build uneven lengths")
    return tuple(lengths)


def rotated_tokens(
    n_tokens: int, num_work_tiles: int, has_segments: int, tile_starts: Optional[Sequence[int]] = None
) -> list[int]:
    """Tokens the reference's tiled kernels rotate (bench_welmv4_inplace_rope_npu.py:
    700-718, 856-867): tile i covers [start_i, start_i + min(64, len_i))."""
    out: list[int] = []
    for tile in range(num_work_tiles):
        if has_segments:
            begin, end = int(tile_starts[tile]), int(tile_starts[tile + 1])
        else:
            begin, end = tile * TILE_TOKENS, min(tile * TILE_TOKENS + TILE_TOKENS, n_tokens)
        count = min(end - begin, TILE_TOKENS)
        out.extend(range(begin, begin + max(count, 0)))
    return out


def tiled_outputs(
    query: torch.Tensor,
    key: torch.Tensor,
    positions: torch.Tensor,
    cache: torch.Tensor,
    num_work_tiles: int,
    has_segments: int,
    tile_starts: Optional[Sequence[int]] = None,
    last_index: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Oracle for an arbitrary tile table: only the tokens the tiles cover
    are rotated (K always; Q rows too in ordinary mode); in mirror mode
    every Q row b < BS is rotated at positions[last_index[b]]."""
    tokens = torch.tensor(rotated_tokens(int(positions.numel()), num_work_tiles, has_segments, tile_starts),
                          dtype=torch.int64)
    k_out = key.clone()
    if tokens.numel():
        k_out[tokens] = apply_reference(key[tokens], positions[tokens], cache)
    if last_index is not None:
        q_out = apply_reference(query, positions.index_select(0, last_index), cache)
    else:
        q_out = query.clone()
        if tokens.numel():
            q_out[tokens] = apply_reference(query[tokens], positions[tokens], cache)
    return q_out, k_out
