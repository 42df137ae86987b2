"""Build recipe for the in-tree sm_100a shared library.

``python -m testfiles_b200.build`` (or ``build_native()``) compiles the
``csrc/*.cu`` translation units with nvcc for ``sm_100a`` only into
``testfiles_b200/libwelm_rope_b200.so``.  The CUDA runtime is linked
statically, so the library loads on a machine without a GPU (the host-only
entry points then work; the device ones report a CUDA error).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
# one translation unit per kernel family; the .cuh headers hold what they share
SOURCES = tuple(CSRC / name for name in (
    "rope_ordinary.cu", "rope_mirror.cu", "rope_kv_write.cu", "rope_tiles.cu", "rope_host_memory.cu",
    "rope_ceiling.cu", "rope_abi.cu"))
HEADERS = (REPO_ROOT / "include" / "welm_rope.h", CSRC / "rope_device.cuh", CSRC / "rope_host.cuh")
LIBRARY = PACKAGE_DIR / "libwelm_rope_b200.so"

NVCC_FLAGS = (
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-Wall",
    "-shared",
)


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(src.stat().st_mtime > built for src in SOURCES + HEADERS)


def build_native(force: bool = False, verbose: bool = False, extra_flags: tuple[str, ...] = ()) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not _stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        _nvcc(), *NVCC_FLAGS, *extra_flags,
        "-I", str(REPO_ROOT / "include"),
        *(str(s) for s in SOURCES),
        "-o", str(tmp),
    ]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, flush=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    args = set(sys.argv[1:])
    path = build_native(force="--force" in args, verbose=True,
                        extra_flags=("-Xptxas", "-v") if "--ptxas-v" in args else ())
    print(path)
