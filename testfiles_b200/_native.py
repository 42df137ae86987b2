"""ctypes binding of the in-tree sm_100a library (``libwelm_rope_b200.so``).

The library is the product: there is no Python or CPU fallback.  Loading
fails loudly when the library is missing; build it with
``python -m testfiles_b200.build``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libwelm_rope_b200.so"

# Status codes (include/welm_rope.h).
OK = 0
ERR_NULL_POINTER = 1
ERR_BAD_MODE = 2
ERR_BAD_SIZE = 3
ERR_BAD_STRIDE = 4
ERR_CAPACITY = 5
ERR_CUDA = 6
ERR_TOO_MANY_TOKENS = 7
ERR_NOT_MAPPED = 8
STATIC_MAX_TOKENS = 2048
LENS_MAX_BATCH = 2048

# Device status bits.
DEV_BAD_POSITION = 1
DEV_BAD_LAST_INDEX = 2
DEV_BAD_TILE = 4
DEV_BAD_LENGTH = 8
DEV_BAD_SLOT = 16
DEV_WAIT_TIMEOUT = 32

_P = ctypes.c_void_p
_I64 = ctypes.c_int64

# name -> (restype, argtypes); every symbol declared in include/welm_rope.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "welm_rope_ordinary": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_mirror": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_mirror_from_lens": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_mirror_kv_write": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                                 _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_build_tiles": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _P, _P, _P]),
    "welm_rope_copy_rope_lanes": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "welm_rope_ordinary_host_static": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_ordinary_mapped": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P]),
    "welm_rope_ceiling_copy": (ctypes.c_int, [_P, _P, _I64, _P]),
    "welm_rope_ceiling_slices": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _P]),
    "welm_rope_ceiling_gather": (ctypes.c_int, [_P, _P, _I64, _I64, _P, _P]),
    "welm_rope_ceiling_tma_slices": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, ctypes.c_int32, ctypes.c_int32, _P,
                                                    _P]),
    "welm_rope_count_tiles_host": (ctypes.c_int, [_P, _I64, _P]),
    "welm_rope_build_tiles_host": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _P]),
    "welm_rope_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "welm_rope_abi_version": (ctypes.c_int, []),
}

ABI_MAJOR = 1  # include/welm_rope.h: WELM_ROPE_ABI_VERSION >> 16
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class WelmRopeError(RuntimeError):
    """A welm_rope entry point returned a non-zero status."""

    def __init__(self, func: str, status: int):
        self.status = status
        super().__init__(f"{func} failed: status {status} ({status_string(status)})")


def load() -> ctypes.CDLL:
    """Load the library once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise RuntimeError(
                    f"{LIBRARY.name} is not built: run `python -m testfiles_b200.build` "
                    "(the sm_100a library is required; there is no fallback)"
                )
            lib = ctypes.CDLL(str(LIBRARY))
            lib.welm_rope_abi_version.restype = ctypes.c_int
            major = lib.welm_rope_abi_version() >> 16
            if major != ABI_MAJOR:
                raise RuntimeError(
                    f"{LIBRARY.name} has ABI major version {major}, these bindings expect {ABI_MAJOR}: "
                    "rebuild it with `python -m testfiles_b200.build`"
                )
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    try:
        raw = load().welm_rope_status_string(int(status))
    except RuntimeError:
        return "library not loaded"
    return raw.decode() if raw else "unknown"


def check(func: str, status: int) -> None:
    if status != OK:
        raise WelmRopeError(func, status)
