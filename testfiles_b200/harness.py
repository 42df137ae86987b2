"""Harness-level drop-in: the reference benchmark's provider table and
``Harness.bind`` (bench_welmv4_inplace_rope_npu.py:922-935, 1088-1100,
1121-1388) over the sm_100a library.

``Harness(device).bind(provider, case, query, key, positions, last_index,
segment_tile_starts)`` checks the mode exactly as the reference does (the
same provider tuples per case, the same ``ValueError`` conditions and
messages, ``KeyError`` for an unknown provider) and returns a zero-argument
launch closure, so the reference's correctness runner and timing loops can
take this harness unchanged.

The provider names are kept; on the B200 each one reaches one of two kernels
with the same tokens rotated as the reference's kernel of that name:

* ``baseline``, ``candidate``, ``generic_prefill`` — the per-token
  semantics: every token, and in mirror modes every Q row ``b < BS`` at
  ``positions[last_index[b]]``: ``rope_prefill`` / ``rope_mirror_prefill``
  with ``has_segments = 0`` over ``ceil(N / 64)`` work tiles;
* ``segmented_prefill``, ``mirror_segmented`` — the segmented tile table
  (``has_segments = 1``);
* ``mirror_contiguous`` — the BS = 1 contiguous mirror.

The reference switches between its per-token and tiled kernels at M = 576 /
640 (bench_welmv4_inplace_rope_npu.py:1324-1338); the B200 kernels gather
positions per token and serve every M, so ``candidate`` needs no threshold.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ops, workloads

PROVIDERS = {
    "baseline": "per-token semantics (rope_prefill / rope_mirror_prefill, has_segments=0)",
    "candidate": "per-token semantics (rope_prefill / rope_mirror_prefill, has_segments=0)",
    "generic_prefill": "per-token semantics over every token (rope_prefill, has_segments=0)",
    "segmented_prefill": "segmented tile table (rope_prefill, has_segments=1)",
    "mirror_contiguous": "BS=1 contiguous KV mirror (rope_mirror_prefill, has_segments=0)",
    "mirror_segmented": "segmented KV mirror (rope_mirror_prefill, has_segments=1)",
}

DEFAULT_PROVIDERS = ("baseline", "candidate")
SEGMENTED_PROVIDERS = ("generic_prefill", "segmented_prefill")
CONTIGUOUS_MIRROR_PROVIDERS = ("baseline", "mirror_contiguous")
SEGMENTED_MIRROR_PROVIDERS = ("baseline", "mirror_segmented")
LEGACY_MIRROR_PROVIDERS = ("baseline",)


def providers_for_case(case: workloads.Case) -> tuple[str, ...]:
    """The providers a case may be bound to (bench_welmv4_inplace_rope_npu.py:1088-1100)."""
    if case.is_segmented_mirror:
        return SEGMENTED_MIRROR_PROVIDERS
    if case.is_segmented:
        return SEGMENTED_PROVIDERS
    if case.is_contiguous_mirror:
        return CONTIGUOUS_MIRROR_PROVIDERS
    if case.phase == "prefill_mirror":
        return LEGACY_MIRROR_PROVIDERS
    return DEFAULT_PROVIDERS


def _tiles(n_tokens: int) -> int:
    return (n_tokens + workloads.TILE_TOKENS - 1) // workloads.TILE_TOKENS


class Harness:
    """Device state shared by every bound launch (bench_welmv4_inplace_rope_npu.py:1121-1162):
    the FP32 cos/sin cache, built once, and the stable placeholder passed as
    the segment pointer of non-segmented launches."""

    def __init__(self, device: torch.device | str = "cuda", seed: int = 20260814,
                 cache: Optional[torch.Tensor] = None) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the harness runs on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.seed = seed
        self.device_index = self.device.index
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.device_name = torch.cuda.get_device_name(self.device)
        if cache is None:
            cache = workloads.make_cos_sin_cache(workloads.REFERENCE_MAX_POSITION, workloads.REFERENCE_ROPE_BASE)
        self.cache = cache.to(self.device, torch.float32).contiguous()
        self.segment_placeholder = ops.segment_placeholder(self.device)

    def metadata(self) -> dict[str, object]:
        return {
            "device": str(self.device),
            "device_name": self.device_name,
            "device_index": self.device_index,
            "num_sms": self.num_sms,
            "torch_version": str(torch.__version__),
            "cuda_version": str(torch.version.cuda),
            "seed": self.seed,
            "dtype": "bfloat16",
            "cache_dtype": "float32",
            "head_dim": ops.HEAD_DIM,
            "rope_dim": ops.ROPE_DIM,
            "num_q_heads": ops.NUM_Q_HEADS,
            "num_k_heads": ops.NUM_K_HEADS,
        }

    def bind(
        self,
        provider: str,
        case: workloads.Case,
        query: torch.Tensor,
        key: torch.Tensor,
        positions: torch.Tensor,
        last_index: Optional[torch.Tensor],
        segment_tile_starts: Optional[torch.Tensor],
    ) -> Callable[[], None]:
        """A launch closure for ``case`` through ``provider`` (bench_welmv4_inplace_rope_npu.py:1164-1388)."""
        n_tokens = int(positions.shape[0])
        batch_size = int(last_index.numel()) if last_index is not None else 0
        q_stride, k_stride = int(query.stride(0)), int(key.stride(0))

        if provider == "mirror_contiguous":
            if not case.is_contiguous_mirror or batch_size != 1:
                raise ValueError("mirror_contiguous requires the isolated BS=1 contiguous mirror cases")
            return self._mirror(query, key, positions, last_index, None, _tiles(n_tokens), n_tokens, batch_size,
                                q_stride, k_stride)

        if case.is_segmented_mirror:
            if segment_tile_starts is None or last_index is None:
                raise ValueError("segmented mirror requires last_index and segment_tile_starts")
            if provider not in SEGMENTED_MIRROR_PROVIDERS:
                raise ValueError(f"unsupported segmented mirror provider: {provider}")
            if provider == "baseline":
                return self._mirror(query, key, positions, last_index, None, _tiles(n_tokens), n_tokens, batch_size,
                                    q_stride, k_stride)
            tiles = int(segment_tile_starts.numel()) - 1
            return self._mirror(query, key, positions, last_index, segment_tile_starts, tiles, n_tokens, batch_size,
                                q_stride, k_stride)

        if case.is_segmented:
            if segment_tile_starts is None:
                raise ValueError("segmented prefill requires segment_tile_starts")
            if provider not in SEGMENTED_PROVIDERS:
                raise ValueError(f"unsupported segmented provider: {provider}")
            if provider == "generic_prefill":
                return self._ordinary(query, key, positions, None, _tiles(n_tokens), n_tokens, q_stride, k_stride)
            tiles = int(segment_tile_starts.numel()) - 1
            return self._ordinary(query, key, positions, segment_tile_starts, tiles, n_tokens, q_stride, k_stride)

        if provider not in PROVIDERS:
            raise KeyError(provider)
        if last_index is not None:  # the per-token kernels' mirror mode
            return self._mirror(query, key, positions, last_index, None, _tiles(n_tokens), n_tokens, batch_size,
                                q_stride, k_stride)
        return self._ordinary(query, key, positions, None, _tiles(n_tokens), n_tokens, q_stride, k_stride)

    def _ordinary(self, query, key, positions, starts, tiles, n_tokens, q_stride, k_stride) -> Callable[[], None]:
        seg = self.segment_placeholder if starts is None else starts
        has_segments = 0 if starts is None else 1
        cache = self.cache

        def launch() -> None:
            ops.rope_prefill(query, key, positions, cache, seg, tiles, n_tokens, q_stride, k_stride, has_segments)

        return launch

    def _mirror(self, query, key, positions, last_index, starts, tiles, n_tokens, batch_size, q_stride,
                k_stride) -> Callable[[], None]:
        seg = self.segment_placeholder if starts is None else starts
        has_segments = 0 if starts is None else 1
        cache = self.cache

        def launch() -> None:
            ops.rope_mirror_prefill(query, key, positions, cache, last_index, seg, tiles, n_tokens, batch_size,
                                    q_stride, k_stride, has_segments)

        return launch
