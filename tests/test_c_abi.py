"""A plain C program as the caller of the C ABI.

tests/c_abi_smoke.c binds include/welm_rope.h the way a C or cgo host would
(no torch; the CUDA runtime only for device and page-locked host memory) and
checks the ordinary, segmented, KV-mirror and mapped-host entries and both
tile builders bit for bit against the C oracle (oracle/rope_oracle.c).  On CPU the program must compile as C99
and link against every symbol it uses; on a B200 it must run and pass.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

from oracle import c_oracle
from testfiles_b200 import _native

REPO = Path(__file__).resolve().parent.parent
SOURCE = REPO / "tests" / "c_abi_smoke.c"


def _cuda_home() -> Path:
    nvcc = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return Path(nvcc).resolve().parent.parent


def build_program(out_dir: Path) -> Path:
    _native.load()  # the library must be built (fails loudly otherwise)
    c_oracle.load()
    cuda = _cuda_home()
    lib_dirs = [str(_native.LIBRARY.parent), str(c_oracle.LIBRARY.parent), str(cuda / "lib64")]
    exe = out_dir / "c_abi_smoke"
    cmd = [
        os.environ.get("CC", "gcc"), "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror",
        "-I", str(REPO / "include"), "-isystem", str(cuda / "include"),
        str(SOURCE), "-o", str(exe),
        f"-L{lib_dirs[0]}", f"-l:{_native.LIBRARY.name}",
        f"-L{lib_dirs[1]}", f"-l:{c_oracle.LIBRARY.name}",
        f"-L{lib_dirs[2]}", "-lcudart",
        *(f"-Wl,-rpath,{d}" for d in lib_dirs),
    ]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_program_compiles_and_links(tmp_path):
    exe = build_program(tmp_path)
    assert exe.exists() and os.access(exe, os.X_OK)


@pytest.mark.gpu
def test_c_program_matches_c_oracle_on_b200(tmp_path):
    exe = build_program(tmp_path)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c-abi ok" in run.stdout
