"""CPU checks of the C ABI: the library loads, exports every declared symbol,
validates arguments on the host before any CUDA call, and its host tile
builder twin matches the reference's tables.  No kernel is launched here."""

from __future__ import annotations

import ctypes
import random
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO
from oracle import rope_oracle
from testfiles_b200 import _native, build
import testfiles_b200 as welm

HEADER = REPO / "include" / "welm_rope.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(welm_rope_\w+)\s*\(", text, flags=re.M))


def test_library_is_built_for_sm100a_only():
    assert build.LIBRARY.exists(), "run python -m testfiles_b200.build"
    assert "arch=compute_100a,code=sm_100a" in build.NVCC_FLAGS


def test_every_declared_symbol_is_exported_and_bound():
    symbols = declared_symbols()
    assert symbols == set(_native.SIGNATURES), symbols ^ set(_native.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", str(build.LIBRARY)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert symbols <= exported, symbols - exported
    lib = _native.load()
    for name in symbols:
        assert getattr(lib, name) is not None


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.welm_rope_abi_version() >> 16 == 1
    header = (REPO / "include" / "welm_rope.h").read_text()
    major, minor = map(int, re.search(r"#define WELM_ROPE_ABI_VERSION \(\((\d+) << 16\) \| (\d+)\)", header).groups())
    assert lib.welm_rope_abi_version() == (major << 16) | minor
    for code in range(9):
        assert _native.status_string(code)
    assert _native.status_string(99) == "unknown welm_rope status"


FAKE = 0x1000  # a non-NULL address; every call below is rejected before it is used


def ordinary(**kw):
    args = dict(q=FAKE, k=FAKE, positions=FAKE, cache=FAKE, starts=None, tiles=1, n=1, qs=1536, ks=256,
                seg=0, maxpos=16, status=None, stream=None)
    args.update(kw)
    return _native.load().welm_rope_ordinary(
        args["q"], args["k"], args["positions"], args["cache"], args["starts"], args["tiles"], args["n"],
        args["qs"], args["ks"], args["seg"], args["maxpos"], args["status"], args["stream"])


def mirror(**kw):
    args = dict(q=FAKE, k=FAKE, positions=FAKE, cache=FAKE, last=FAKE, starts=None, tiles=1, n=1, bs=1,
                qs=1536, ks=256, seg=0, maxpos=16, status=None, stream=None)
    args.update(kw)
    return _native.load().welm_rope_mirror(
        args["q"], args["k"], args["positions"], args["cache"], args["last"], args["starts"], args["tiles"],
        args["n"], args["bs"], args["qs"], args["ks"], args["seg"], args["maxpos"], args["status"],
        args["stream"])


def test_host_validation_ordinary():
    assert ordinary(seg=2) == _native.ERR_BAD_MODE
    assert ordinary(seg=-1) == _native.ERR_BAD_MODE
    assert ordinary(n=-1) == _native.ERR_BAD_SIZE
    assert ordinary(tiles=-3) == _native.ERR_BAD_SIZE
    assert ordinary(maxpos=-1) == _native.ERR_BAD_SIZE
    assert ordinary(n=1 << 40, tiles=1 << 34) == _native.ERR_BAD_SIZE
    assert ordinary(q=None) == _native.ERR_NULL_POINTER
    assert ordinary(cache=None) == _native.ERR_NULL_POINTER
    assert ordinary(seg=1, starts=None) == _native.ERR_NULL_POINTER
    assert ordinary(n=4, tiles=1, qs=1535) == _native.ERR_BAD_STRIDE
    assert ordinary(n=4, tiles=1, ks=255) == _native.ERR_BAD_STRIDE
    # zero work is a no-op that needs no pointers and launches nothing
    assert ordinary(q=None, k=None, positions=None, cache=None, n=0) == _native.OK
    assert ordinary(q=None, k=None, positions=None, cache=None, tiles=0) == _native.OK


def test_host_validation_mirror():
    assert mirror(seg=3) == _native.ERR_BAD_MODE
    assert mirror(bs=-1) == _native.ERR_BAD_SIZE
    assert mirror(last=None) == _native.ERR_NULL_POINTER
    assert mirror(k=None) == _native.ERR_NULL_POINTER
    assert mirror(q=None, bs=1) == _native.ERR_NULL_POINTER
    assert mirror(bs=2, qs=100) == _native.ERR_BAD_STRIDE
    assert mirror(n=2, ks=8) == _native.ERR_BAD_STRIDE
    assert mirror(seg=1, starts=None) == _native.ERR_NULL_POINTER
    assert mirror(q=None, k=None, positions=None, cache=None, last=None, n=0, bs=0) == _native.OK


def test_host_validation_device_builder():
    lib = _native.load()
    assert lib.welm_rope_build_tiles(FAKE, -1, FAKE, 8, FAKE, None, None, None) == _native.ERR_BAD_SIZE
    assert lib.welm_rope_build_tiles(FAKE, 2, FAKE, 0, FAKE, None, None, None) == _native.ERR_CAPACITY
    assert lib.welm_rope_build_tiles(None, 2, FAKE, 8, FAKE, None, None, None) == _native.ERR_NULL_POINTER
    assert lib.welm_rope_build_tiles(FAKE, 2, None, 8, FAKE, None, None, None) == _native.ERR_NULL_POINTER
    assert lib.welm_rope_build_tiles(FAKE, 2, FAKE, 8, None, None, None, None) == _native.ERR_NULL_POINTER


def test_host_builder_matches_reference_tables(tile_tables):
    for name, rec in tile_tables.items():
        starts, tiles, last = welm.build_segment_tile_starts(rec["segment_lens"])
        assert starts.tolist() == rec["segment_tile_starts"], name
        assert tiles == len(rec["segment_tile_starts"]) - 1
        if rec["last_index"] is not None:
            assert last.tolist() == rec["last_index"], name


def test_host_builder_random_lengths_match_oracle():
    rng = random.Random(7)
    for _ in range(200):
        bs = rng.randint(0, 40)
        lens = [rng.choice([0, 1, 2, 63, 64, 65, 127, 128, 129, rng.randint(0, 3000)]) for _ in range(bs)]
        starts, tiles, last = welm.build_segment_tile_starts(lens)
        assert starts.tolist() == rope_oracle.build_tile_starts(lens)
        assert tiles == sum((x + 63) // 64 for x in lens) == welm.count_segment_tiles(lens)
        if bs and sum(lens):
            assert last.tolist() == list(np.cumsum(lens) - 1)


def test_host_builder_errors():
    lib = _native.load()
    lens = np.array([5, -1], dtype=np.int64)
    with pytest.raises(welm.WelmRopeError):
        welm.count_segment_tiles(lens)
    good = np.array([65, 1], dtype=np.int64)
    out = np.zeros(3, dtype=np.int32)
    tiles = ctypes.c_int64(0)
    rc = lib.welm_rope_build_tiles_host(good.ctypes.data, 2, out.ctypes.data, 3, ctypes.byref(tiles), None)
    assert rc == _native.ERR_CAPACITY  # needs T + 1 = 4 slots
    out = np.zeros(4, dtype=np.int32)
    rc = lib.welm_rope_build_tiles_host(good.ctypes.data, 2, out.ctypes.data, 4, ctypes.byref(tiles), None)
    assert rc == _native.OK and out.tolist() == [0, 64, 65, 66] and tiles.value == 3
    empty = welm.build_segment_tile_starts([])
    assert empty[0].tolist() == [0] and empty[1] == 0 and empty[2].numel() == 0


def test_launcher_case_selection_and_fields():
    from testfiles_b200 import launcher, workloads

    assert len(launcher.select_cases("decode")) == 128
    assert len(launcher.select_cases("reference")) == 193
    cases = launcher.select_cases("b_prefill_m16384,mirror_segmented_m16384_b128_uneven")
    assert [c.name for c in cases] == ["b_prefill_m16384", "mirror_segmented_m16384_b128_uneven"]
    fields = launcher.case_fields(cases[1])
    assert fields["path"] == "kv_mirror" and fields["has_segments"] == 1 and fields["batch_size"] == 128
    assert workloads.min_bytes(cases[0]) == 2056 * 16384
    assert workloads.min_bytes(cases[1]) == 520 * 16384 + 1544 * 128 + 4 * 321


def test_copy_rope_lanes_host_validation():
    lib = _native.load()
    assert lib.welm_rope_copy_rope_lanes(FAKE, FAKE, -1, 6, 1536, 1536, 0, None) == _native.ERR_BAD_SIZE
    assert lib.welm_rope_copy_rope_lanes(FAKE, FAKE, 4, 6, 1536, 1536, 2, None) == _native.ERR_BAD_MODE
    assert lib.welm_rope_copy_rope_lanes(None, FAKE, 4, 6, 1536, 1536, 0, None) == _native.ERR_NULL_POINTER
    assert lib.welm_rope_copy_rope_lanes(FAKE, FAKE, 4, 6, 1000, 1536, 0, None) == _native.ERR_BAD_STRIDE
    assert lib.welm_rope_copy_rope_lanes(None, None, 0, 6, 0, 0, 0, None) == _native.OK


def test_host_entry_rejects_misuse():
    import torch
    from testfiles_b200 import host

    q = torch.zeros((4, 6, 256), dtype=torch.bfloat16)
    k = torch.zeros((4, 1, 256), dtype=torch.bfloat16)
    pos = torch.zeros(4, dtype=torch.int64)
    cache = torch.zeros((8, 64), dtype=torch.float32)
    with pytest.raises(ValueError):  # the cache selects the device and must be on one
        host.welmv4_inplace_rope_host(q, k, pos, cache)
    assert host.lane_bytes(16384) == (16384 * 7 * 128 + 16384 * 8, 16384 * 7 * 128)


def test_static_host_entry_rejects_oversized_batches_before_any_cuda_call():
    lib = _native.load()
    rc = lib.welm_rope_ordinary_host_static(FAKE, FAKE, FAKE, FAKE, _native.STATIC_MAX_TOKENS + 1, 1536, 256, 16,
                                            None, None)
    assert rc == _native.ERR_TOO_MANY_TOKENS
    assert "2048" in _native.status_string(rc)
    assert lib.welm_rope_ordinary_host_static(FAKE, FAKE, FAKE, FAKE, -1, 1536, 256, 16, None, None) == \
        _native.ERR_BAD_SIZE
    assert lib.welm_rope_ordinary_host_static(None, FAKE, FAKE, FAKE, 4, 1536, 256, 16, None, None) == \
        _native.ERR_NULL_POINTER
    assert lib.welm_rope_ordinary_host_static(None, None, None, None, 0, 0, 0, 0, None, None) == _native.OK


def test_mirror_from_lens_host_validation():
    lib = _native.load()
    args = lambda **kw: [kw.get(n, d) for n, d in (("q", FAKE), ("k", FAKE), ("p", FAKE), ("c", FAKE), ("l", FAKE),
                                                   ("n", 16), ("bs", 2), ("qs", 1536), ("ks", 256), ("mp", 16),
                                                   ("st", None), ("s", None))]
    f = lib.welm_rope_mirror_from_lens
    assert f(*args(bs=_native.LENS_MAX_BATCH + 1)) == _native.ERR_BAD_SIZE
    assert f(*args(n=-1)) == _native.ERR_BAD_SIZE
    assert f(*args(l=None)) == _native.ERR_NULL_POINTER
    assert f(*args(l=FAKE + 4)) == _native.ERR_BAD_STRIDE  # lengths must be 8-byte aligned
    assert f(*args(bs=2, qs=8)) == _native.ERR_BAD_STRIDE
    assert f(*args(q=None, k=None, p=None, c=None, l=None, bs=0)) == _native.OK


def test_kv_write_host_validation():
    lib = _native.load()
    base = dict(q=FAKE, qo=FAKE, k=FAKE, v=FAKE, p=FAKE, c=FAKE, li=FAKE, sl=FAKE, kc=FAKE, vc=FAKE, n=8, bs=2,
                qs=1536, qos=1536, ks=256, vs=256, css=256, ns=64, mp=16)
    order = ("q", "qo", "k", "v", "p", "c", "li", "sl", "kc", "vc", "n", "bs", "qs", "qos", "ks", "vs", "css", "ns", "mp")
    f = lambda **kw: lib.welm_rope_mirror_kv_write(*[{**base, **kw}[x] for x in order], None, None)
    assert f(n=-1) == _native.ERR_BAD_SIZE
    assert f(sl=None) == _native.ERR_NULL_POINTER
    assert f(v=None) == _native.ERR_NULL_POINTER  # v and value_cache come together
    assert f(qo=None) == _native.ERR_NULL_POINTER
    assert f(css=100) == _native.ERR_BAD_STRIDE
    assert f(k=FAKE + 2) == _native.ERR_BAD_STRIDE  # 16-byte alignment required
    assert f(q=None, qo=None, k=None, v=None, p=None, c=None, li=None, sl=None, kc=None, vc=None, n=0) == _native.OK


def test_mapped_entry_host_validation():
    """Refusals happen on the host before any launch; FAKE pointers are never
    reachable by a device, so even valid sizes end in ERR_NOT_MAPPED."""
    lib = _native.load()
    call = lib.welm_rope_ordinary_mapped
    assert call(FAKE, FAKE, FAKE, FAKE, -1, 1536, 256, 16, None, None) == _native.ERR_BAD_SIZE
    assert call(FAKE, FAKE, FAKE, FAKE, 4, 1536, 256, -1, None, None) == _native.ERR_BAD_SIZE
    assert call(None, None, None, None, 0, 0, 0, 0, None, None) == _native.OK
    assert call(None, FAKE, FAKE, FAKE, 4, 1536, 256, 16, None, None) == _native.ERR_NULL_POINTER
    assert call(FAKE, FAKE, None, FAKE, 4, 1536, 256, 16, None, None) == _native.ERR_NULL_POINTER
    assert call(FAKE, FAKE, FAKE, FAKE, 4, 1535, 256, 16, None, None) == _native.ERR_BAD_STRIDE
    assert call(FAKE, FAKE, FAKE, FAKE, 4, 1540, 256, 16, None, None) == _native.ERR_BAD_STRIDE  # not 8-aligned
    assert call(FAKE + 2, FAKE, FAKE, FAKE, 4, 1536, 256, 16, None, None) == _native.ERR_BAD_STRIDE
    assert call(FAKE, FAKE, FAKE, FAKE + 4, 4, 1536, 256, 16, None, None) == _native.ERR_BAD_STRIDE
    assert call(FAKE, FAKE, FAKE, FAKE, 4, 1536, 256, 16, None, None) == _native.ERR_NOT_MAPPED
    assert "page-locked" in _native.status_string(_native.ERR_NOT_MAPPED)


def test_host_entry_transport_argument():
    import torch
    from testfiles_b200 import host

    q = torch.zeros((2, 6, 256), dtype=torch.bfloat16)
    k = torch.zeros((2, 1, 256), dtype=torch.bfloat16)
    pos = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(ValueError, match="transport"):
        host.welmv4_inplace_rope_host(q, k, pos, torch.zeros((8, 64)), transport="zero-copy")


def test_launcher_csv_writer(tmp_path):
    import csv

    from testfiles_b200 import launcher

    recs = [{"record_type": "timing", "case": "a", "us_per_launch": 1.5, "clocks": {"sm_mhz": 1965}},
            {"record_type": "launch", "case": "b", "iters": 3}]
    path = tmp_path / "records.csv"
    launcher.write_csv(recs, str(path))
    rows = list(csv.DictReader(path.open()))
    assert [r["case"] for r in rows] == ["a", "b"]
    assert list(rows[0]) == ["record_type", "case", "us_per_launch", "clocks", "iters"]
    assert rows[0]["clocks"] == '{"sm_mhz": 1965}' and rows[1]["us_per_launch"] == ""


def test_clock_sampler_without_a_device_reports_no_samples():
    from testfiles_b200.clocks import ClockSampler

    with ClockSampler(0) as s:
        pass
    summary = s.summary()
    assert summary["samples"] == 0 or summary["sm_mhz"] is not None


def test_bindings_match_the_header_abi_major():
    header = (REPO / "include" / "welm_rope.h").read_text()
    major = int(re.search(r"#define WELM_ROPE_ABI_VERSION \(\((\d+) << 16\)", header).group(1))
    assert _native.ABI_MAJOR == major


def test_ceiling_entries_host_validation():
    """The measurement kernels refuse bad sizes, NULL and misaligned buffers
    on the host; only valid calls would reach a launch (none here)."""
    lib = _native.load()
    copy, slices = lib.welm_rope_ceiling_copy, lib.welm_rope_ceiling_slices
    assert copy(FAKE, FAKE, -16, None) == _native.ERR_BAD_SIZE
    assert copy(FAKE, FAKE, 24, None) == _native.ERR_BAD_SIZE  # not a multiple of 16
    assert copy(None, None, 0, None) == _native.OK
    assert copy(None, FAKE, 16, None) == _native.ERR_NULL_POINTER
    assert copy(FAKE + 8, FAKE, 16, None) == _native.ERR_BAD_STRIDE
    assert slices(FAKE, FAKE, -1, 1536, 256, None) == _native.ERR_BAD_SIZE
    assert slices(None, None, 0, 0, 0, None) == _native.OK
    assert slices(FAKE, None, 4, 1536, 256, None) == _native.ERR_NULL_POINTER
    assert slices(FAKE, FAKE, 4, 1535, 256, None) == _native.ERR_BAD_STRIDE
    assert slices(FAKE, FAKE, 4, 1540, 256, None) == _native.ERR_BAD_STRIDE  # not 8-aligned
    assert slices(FAKE, FAKE + 2, 4, 1536, 256, None) == _native.ERR_BAD_STRIDE
    gather = lib.welm_rope_ceiling_gather
    assert gather(FAKE, FAKE, -1, 64, None, None) == _native.ERR_BAD_SIZE
    assert gather(FAKE, FAKE, 4, -1, None, None) == _native.ERR_BAD_SIZE
    assert gather(None, None, 0, 64, None, None) == _native.OK
    assert gather(None, FAKE, 4, 64, None, None) == _native.ERR_NULL_POINTER
    assert gather(FAKE, FAKE + 8, 4, 64, None, None) == _native.ERR_BAD_STRIDE  # the cache is read in 16-byte vectors
    tma = lib.welm_rope_ceiling_tma_slices
    assert tma(FAKE, FAKE, -1, 1536, 256, 0, 4, None, None) == _native.ERR_BAD_SIZE
    assert tma(FAKE, FAKE, 1 << 31, 1536, 256, 0, 4, None, None) == _native.ERR_BAD_SIZE
    assert tma(FAKE, FAKE, 4, 1536, 256, -1, 4, None, None) == _native.ERR_BAD_SIZE
    assert tma(FAKE, FAKE, 4, 1536, 256, 0, 3, None, None) == _native.ERR_BAD_MODE  # 2, 4 or 6 stages
    assert tma(None, None, 0, 0, 0, 0, 2, None, None) == _native.OK
    assert tma(None, FAKE, 4, 1536, 256, 0, 2, None, None) == _native.ERR_NULL_POINTER
    assert tma(FAKE, FAKE, 1, 0, 0, 0, 2, None, None) == _native.ERR_BAD_STRIDE  # tensor maps need whole rows
    assert tma(FAKE, FAKE, 4, 1540, 256, 0, 2, None, None) == _native.ERR_BAD_STRIDE
    assert tma(FAKE + 8, FAKE, 4, 1536, 256, 0, 2, None, None) == _native.ERR_BAD_STRIDE


def test_device_status_bits_match_the_header():
    header = (REPO / "include" / "welm_rope.h").read_text()
    bits = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define WELM_ROPE_DEV_(\w+) (\d+)", header)}
    assert bits == {name[len("DEV_"):]: getattr(_native, name) for name in dir(_native) if name.startswith("DEV_")}


def test_launcher_rejects_fewer_than_one_buffer_set():
    import torch

    from testfiles_b200 import launcher, workloads

    with pytest.raises(SystemExit):
        launcher.main(["--time", "--sets", "0"])
    with pytest.raises(ValueError, match="sets"):
        launcher.time_case(workloads.find_case("b_decode_m1"), torch.device("cpu"), sets=0)


def test_launcher_kernel_names_follow_the_head_split_rule():
    from testfiles_b200 import launcher, workloads

    src = (REPO / "testfiles_b200" / "csrc" / "rope_host.cuh").read_text()
    limit = int(re.search(r"constexpr int64_t kHeadSplitMaxTokens = (\d+);", src).group(1))
    assert launcher.HEAD_SPLIT_MAX_TOKENS == limit
    assert launcher.kernel_name(workloads.find_case("b_decode_m1")) == "rope_ordinary_head_kernel"
    assert launcher.kernel_name(workloads.find_case("b_prefill_m3328")) == "rope_ordinary_head_kernel"
    assert launcher.kernel_name(workloads.find_case("b_prefill_m3329")) == "rope_ordinary_stream_kernel"
    assert launcher.kernel_name(workloads.find_case("segmented_m4096_b8_aligned")) == "rope_ordinary_stream_kernel"
    sparse = workloads.Case("sparse", "segmented_prefill", 4096, 129, (1,) * 128 + (3968,))
    assert launcher.kernel_name(sparse) == "rope_ordinary_kernel"  # 190 tiles, 4096 tokens: under half the slots
    assert launcher.kernel_name(workloads.find_case("b_mirror_contiguous_n8192")) == "rope_mirror_head_kernel"
