"""B200-native (sm_100a) WeLMv4 in-place partial rotary embedding.

A drop-in for the reference's ``welmv4_inplace_rope_npu`` op (ordinary
prefill / decode and KV-mirror prefill, contiguous or segmented) backed by
hand-written CUDA in ``libwelm_rope_b200.so`` called through its C ABI
(``include/welm_rope.h``).  There is no CPU fallback.
"""

from .ops import (  # noqa: F401
    HEAD_DIM,
    NUM_K_HEADS,
    NUM_Q_HEADS,
    ROPE_DIM,
    TILE_TOKENS,
    WelmRopeError,
    build_segment_tile_starts,
    build_segment_tile_starts_device,
    count_segment_tiles,
    rope_mirror_from_lens,
    rope_mirror_kv_write,
    rope_mirror_prefill,
    rope_prefill,
    segment_placeholder,
    welmv4_inplace_rope,
    welmv4_inplace_rope_npu,
)
from .host import welmv4_inplace_rope_host  # noqa: F401,E402
from .harness import Harness, providers_for_case  # noqa: F401,E402

__version__ = "0.1.0"
