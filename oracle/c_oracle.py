"""ctypes loader of the C restatement (rope_oracle.c) — TEST INFRASTRUCTURE ONLY.

The library is built by ``make -C oracle`` (``__graft_entry__.build()`` does
it; :func:`load` builds it on first use when gcc is available).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path
from typing import Optional, Sequence

import torch

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "librope_oracle.so"
_lib: Optional[ctypes.CDLL] = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists() or LIBRARY.stat().st_mtime < (HERE / "rope_oracle.c").stat().st_mtime:
            build()
        lib = ctypes.CDLL(str(LIBRARY))
        p, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.welm_oracle_apply.argtypes = [p, p, i64, i64, i64, p, p, i64]
        lib.welm_oracle_apply.restype = i64
        lib.welm_oracle_count_tiles.argtypes = [p, i64]
        lib.welm_oracle_count_tiles.restype = i64
        lib.welm_oracle_build_tiles.argtypes = [p, i64, p]
        lib.welm_oracle_build_tiles.restype = i64
        _lib = lib
    return _lib


def apply(data: torch.Tensor, rope_positions: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
    """C restatement of apply_reference on CPU tensors [rows, heads, 256]."""
    data = data.contiguous()
    out = torch.empty_like(data)
    pos = rope_positions.to(torch.int64).contiguous()
    cache = cache.to(torch.float32).contiguous()
    rows, heads = data.shape[0], data.shape[1]
    load().welm_oracle_apply(data.data_ptr() or None, out.data_ptr() or None, rows, heads, heads * 256,
                             pos.data_ptr() or None, cache.data_ptr() or None, cache.shape[0])
    return out


def reference_outputs(query, key, positions, last_index, cache) -> tuple[torch.Tensor, torch.Tensor]:
    q_pos = positions if last_index is None else positions.index_select(0, last_index)
    return apply(query, q_pos, cache), apply(key, positions, cache)


def build_tiles(lens: Sequence[int]) -> list[int]:
    arr = (ctypes.c_int64 * max(1, len(lens)))(*lens)
    n = load().welm_oracle_count_tiles(arr, len(lens))
    starts = (ctypes.c_int32 * (n + 1))()
    load().welm_oracle_build_tiles(arr, len(lens), starts)
    return list(starts)
