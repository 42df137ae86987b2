"""Workload catalogue and seeded synthetic inputs for the in-place RoPE.

Two input flavours exist for every case:

* ``"reference"`` reproduces the reference benchmark's generators
  (bench_welmv4_inplace_rope_npu.py:1391-1486): cache base 1e5 with 32768
  rows, per-case seed ``seed + 17*N + 101*BS``, prefill positions starting at
  113, segmented positions ``113 + 97*request + local``, decode / legacy
  mirror positions ``(17 i + 11) % 32768``.  Used to pin parity against the
  reference's own outputs.
* ``"baseline"`` is the benchmark's own configuration set: cache base
  1e4 with 16384 rows, prefill positions ``0..M-1``, decode positions uniform
  in [0, 16383], segmented positions restarting at 0 in every request,
  seeded-uneven request lengths drawn as a uniform partition (lengths >= 1).

Random Q/K are drawn on the CPU (``torch.manual_seed`` + ``torch.randn`` in
BF16, the reference's draw order: Q then K) and then moved to the target
device, so the same seed gives the same tensors on every machine.

The case table mirrors the reference catalogue (bench_welmv4_inplace_rope_npu.py:
78-288): decode M=1..128, 46 prefill sizes, 2 legacy mirror cases, 4 BS=1
contiguous mirror cases, 7 segmented mirror cases, 6 segmented prefill
cases (193 in all).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

HEAD_DIM = 256
ROPE_DIM = 64
NUM_Q_HEADS = 6
NUM_K_HEADS = 1
TILE_TOKENS = 64

REFERENCE_SEED = 20260814
REFERENCE_MAX_POSITION = 32768
REFERENCE_ROPE_BASE = 100000.0
REFERENCE_POSITION_START = 113
BENCH_SEED = 20261201
BENCH_MAX_POSITION = 16384
BENCH_ROPE_BASE = 10000.0

PHASES = (
    "decode",
    "prefill",
    "segmented_prefill",
    "prefill_mirror",
    "prefill_mirror_contiguous",
    "prefill_mirror_segmented",
)


@dataclass(frozen=True)
class Case:
    """One workload: phase, token count N, request count BS, request lengths."""

    name: str
    phase: str
    n_tokens: int
    batch_size: int = 0
    segment_lens: tuple[int, ...] = ()
    flavour: str = "reference"

    def __post_init__(self) -> None:
        if self.phase not in PHASES:
            raise ValueError(f"unknown phase {self.phase}")
        if self.segment_lens and sum(self.segment_lens) != self.n_tokens:
            raise ValueError(f"{self.name}: segment lengths sum to {sum(self.segment_lens)}, not {self.n_tokens}")

    @property
    def is_mirror(self) -> bool:
        return self.phase.startswith("prefill_mirror")

    @property
    def is_contiguous_mirror(self) -> bool:
        return self.phase == "prefill_mirror_contiguous"

    @property
    def is_segmented_mirror(self) -> bool:
        return self.phase == "prefill_mirror_segmented"

    @property
    def is_segmented(self) -> bool:
        return bool(self.segment_lens)

    @property
    def request_count(self) -> int:
        return len(self.segment_lens)

    @property
    def q_rows(self) -> int:
        return self.batch_size if self.is_mirror else self.n_tokens


@dataclass
class Inputs:
    """Device (or CPU) tensors of one case plus the launch integers."""

    query: torch.Tensor
    key: torch.Tensor
    positions: torch.Tensor
    cache: torch.Tensor
    last_index: Optional[torch.Tensor] = None
    segment_tile_starts: Optional[torch.Tensor] = None
    num_work_tiles: int = 0
    has_segments: int = 0
    extra: dict = field(default_factory=dict)

    def to(self, device: torch.device | str) -> "Inputs":
        mv = lambda t: None if t is None else t.to(device)  # noqa: E731
        return Inputs(mv(self.query), mv(self.key), mv(self.positions), mv(self.cache), mv(self.last_index),
                      mv(self.segment_tile_starts), self.num_work_tiles, self.has_segments, dict(self.extra))

    def clone(self) -> "Inputs":
        out = self.to(self.query.device)
        out.query = self.query.clone()
        out.key = self.key.clone()
        return out


# ---------------------------------------------------------------------------
# Small helpers (product-side copies; the oracle restates them separately).
# ---------------------------------------------------------------------------
def make_cos_sin_cache(max_position: int, base: float, rope_dim: int = ROPE_DIM,
                       device: torch.device | str = "cpu") -> torch.Tensor:
    """FP32 [max_position, rope_dim]: cos(p * f_i) then sin(p * f_i),
    f_i = base ** -(2 i / rope_dim); computed on the CPU, then moved."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rope_dim, 2, dtype=torch.float32) / rope_dim))
    freqs = torch.outer(torch.arange(max_position, dtype=torch.float32), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(device=device, dtype=torch.float32)


def tile_starts_for(lens: tuple[int, ...]) -> list[int]:
    starts: list[int] = []
    token = 0
    for length in lens:
        starts.extend(range(token, token + length, TILE_TOKENS))
        token += length
    starts.append(token)
    return starts


def reference_uneven_lens(total: int, batch_size: int) -> tuple[int, ...]:
    """The reference's deterministic uneven pattern (bench_welmv4_inplace_rope_npu.py:115-122)."""
    pattern = (-31, -17, -9, -1, 1, 9, 17, 31)
    base = total // batch_size
    lengths = [base + pattern[i % len(pattern)] for i in range(batch_size)]
    lengths[-1] += total - sum(lengths)
    assert min(lengths) > 0 and sum(lengths) == total
    return tuple(lengths)


def seeded_uneven_lens(total: int, batch_size: int, seed: int) -> tuple[int, ...]:
    """Uniform random partition of ``total`` into ``batch_size`` lengths >= 1."""
    if batch_size <= 0 or batch_size > total:
        raise ValueError("need 1 <= batch_size <= total")
    rng = np.random.default_rng(seed)
    cuts = np.sort(rng.choice(np.arange(1, total), size=batch_size - 1, replace=False)) if batch_size > 1 else []
    edges = [0, *[int(c) for c in cuts], total]
    return tuple(edges[i + 1] - edges[i] for i in range(batch_size))


# ---------------------------------------------------------------------------
# Catalogues.
# ---------------------------------------------------------------------------
PREFILL_SIZES = (
    128, 256, 448, 449, 512, 576, 577, 640, 641, 768, 769, 896, 897, 960, 961, 1024, 1025,
    1152, 1153, 1280, 1281, 1536, 2048, 2049, 2304, 2305, 2560, 2561, 2816, 2817, 3072, 3073,
    3328, 3329, 3584, 3585, 3840, 3841, 4096, 4097, 6145, 7169, 8191, 8192, 9616, 16384,
)


def reference_cases() -> tuple[Case, ...]:
    """The reference's 193-case catalogue (bench_welmv4_inplace_rope_npu.py:126-288)."""
    decode = tuple(Case(f"decode_m{m}", "decode", m) for m in range(1, 129))
    prefill = tuple(Case(f"prefill_m{m}", "prefill", m) for m in PREFILL_SIZES)
    legacy = (Case("mirror_m8192_bs4", "prefill_mirror", 8192, 4),
              Case("mirror_m16384_bs8", "prefill_mirror", 16384, 8))
    contiguous = tuple(Case(f"mirror_contiguous_m{m}_bs1", "prefill_mirror_contiguous", m, 1)
                       for m in (8192, 9616, 16361, 16384))
    uneven_9616 = (1025, 1151, 1183, 1201, 1217, 1231, 1267, 1341)
    seg_mirror = (
        Case("mirror_segmented_m8192_b2_aligned", "prefill_mirror_segmented", 8192, 2, (4096,) * 2),
        Case("mirror_segmented_m8192_b4_aligned", "prefill_mirror_segmented", 8192, 4, (2048,) * 4),
        Case("mirror_segmented_m9616_b8_uneven", "prefill_mirror_segmented", 9616, 8, uneven_9616),
        Case("mirror_segmented_m8192_b16_aligned", "prefill_mirror_segmented", 8192, 16, (512,) * 16),
        Case("mirror_segmented_m16384_b32_aligned", "prefill_mirror_segmented", 16384, 32, (512,) * 32),
        Case("mirror_segmented_m16384_b64_aligned", "prefill_mirror_segmented", 16384, 64, (256,) * 64),
        Case("mirror_segmented_m16384_b128_uneven", "prefill_mirror_segmented", 16384, 128,
             reference_uneven_lens(16384, 128)),
    )
    seg_prefill = (
        Case("segmented_m4096_b8_aligned", "segmented_prefill", 4096, segment_lens=(512,) * 8),
        Case("segmented_m8192_b32_aligned", "segmented_prefill", 8192, segment_lens=(256,) * 32),
        Case("segmented_m9616_b8_uneven", "segmented_prefill", 9616, segment_lens=uneven_9616),
        Case("segmented_m16384_b8_uneven", "segmented_prefill", 16384,
             segment_lens=(1025, 1537, 1793, 2047, 2113, 2305, 2559, 3005)),
        Case("segmented_m16384_b64_aligned", "segmented_prefill", 16384, segment_lens=(256,) * 64),
        Case("segmented_m16384_b128_uneven", "segmented_prefill", 16384,
             segment_lens=reference_uneven_lens(16384, 128)),
    )
    return decode + prefill + legacy + contiguous + seg_mirror + seg_prefill


def baseline_cases(include_sweeps: bool = True) -> tuple[Case, ...]:
    """The benchmark configurations: M=8192 prefill, decode M=1..128, the
    prefill sweep with tails, BS=1 contiguous mirror for N in {8192, 9616,
    16361, 16384}, and segmented mirror for N in {8192, 9616, 16384} x BS in
    {2..128}, equal (64-aligned) or seeded-uneven lengths."""
    out: list[Case] = [Case("b_prefill_m8192", "prefill", 8192, flavour="baseline")]
    if include_sweeps:
        out += [Case(f"b_decode_m{m}", "decode", m, flavour="baseline") for m in range(1, 129)]
        out += [Case(f"b_prefill_m{m}", "prefill", m, flavour="baseline") for m in PREFILL_SIZES if m != 8192]
    out += [Case(f"b_mirror_contiguous_n{n}", "prefill_mirror_contiguous", n, 1, flavour="baseline")
            for n in (8192, 9616, 16361, 16384)]
    for n in (8192, 9616, 16384):
        for bs in (2, 4, 8, 16, 32, 64, 128):
            if n % bs == 0 and (n // bs) % TILE_TOKENS == 0:
                out.append(Case(f"b_mirror_segmented_n{n}_bs{bs}_aligned", "prefill_mirror_segmented", n, bs,
                                (n // bs,) * bs, flavour="baseline"))
            lens = seeded_uneven_lens(n, bs, BENCH_SEED + 31 * n + bs)
            out.append(Case(f"b_mirror_segmented_n{n}_bs{bs}_uneven", "prefill_mirror_segmented", n, bs, lens,
                            flavour="baseline"))
    return tuple(out)


def find_case(name: str) -> Case:
    for case in reference_cases() + baseline_cases():
        if case.name == name:
            return case
    raise KeyError(name)


# ---------------------------------------------------------------------------
# Input generation.
# ---------------------------------------------------------------------------
_CACHE_MEMO: dict[tuple[int, float], torch.Tensor] = {}


def cache_for(flavour: str) -> torch.Tensor:
    key = ((REFERENCE_MAX_POSITION, REFERENCE_ROPE_BASE) if flavour == "reference"
           else (BENCH_MAX_POSITION, BENCH_ROPE_BASE))
    if key not in _CACHE_MEMO:
        _CACHE_MEMO[key] = make_cos_sin_cache(*key)
    return _CACHE_MEMO[key]


def _positions(case: Case) -> torch.Tensor:
    n = case.n_tokens
    if case.flavour == "reference":
        if case.is_segmented:
            chunks = [torch.arange(length, dtype=torch.int64) + REFERENCE_POSITION_START + 97 * r
                      for r, length in enumerate(case.segment_lens)]
            return torch.cat(chunks) if chunks else torch.empty(0, dtype=torch.int64)
        if case.phase in ("prefill", "prefill_mirror_contiguous"):
            return torch.arange(n, dtype=torch.int64) + REFERENCE_POSITION_START
        return (torch.arange(n, dtype=torch.int64) * 17 + 11) % REFERENCE_MAX_POSITION
    # baseline flavour
    if case.is_segmented:
        chunks = [torch.arange(length, dtype=torch.int64) for length in case.segment_lens]
        return torch.cat(chunks) if chunks else torch.empty(0, dtype=torch.int64)
    if case.phase == "decode":
        rng = np.random.default_rng(BENCH_SEED + 7 * n)
        return torch.from_numpy(rng.integers(0, BENCH_MAX_POSITION, size=n, dtype=np.int64))
    if case.phase == "prefill_mirror":
        return (torch.arange(n, dtype=torch.int64) * 17 + 11) % BENCH_MAX_POSITION
    return torch.arange(n, dtype=torch.int64)


def _last_index(case: Case) -> Optional[torch.Tensor]:
    if not case.is_mirror:
        return None
    if case.is_segmented:
        values = np.cumsum(np.asarray(case.segment_lens, dtype=np.int64)) - 1
        return torch.from_numpy(values.astype(np.int64))
    n, bs = case.n_tokens, case.batch_size
    return torch.tensor([max(0, min(n - 1, (i + 1) * n // bs - 1)) for i in range(bs)], dtype=torch.int64)


def case_seed(case: Case, seed: Optional[int] = None) -> int:
    if seed is None:
        seed = REFERENCE_SEED if case.flavour == "reference" else BENCH_SEED
    return seed + case.n_tokens * 17 + case.batch_size * 101


def make_inputs(case: Case, device: torch.device | str = "cpu", seed: Optional[int] = None) -> Inputs:
    """Seeded inputs of ``case`` (drawn on the CPU, then moved to ``device``)."""
    positions = _positions(case)
    gen = torch.Generator(device="cpu")
    gen.manual_seed(case_seed(case, seed))
    query = torch.randn((case.q_rows, NUM_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, generator=gen)
    key = torch.randn((case.n_tokens, NUM_K_HEADS, HEAD_DIM), dtype=torch.bfloat16, generator=gen)
    starts = None
    tiles = (case.n_tokens + TILE_TOKENS - 1) // TILE_TOKENS
    if case.is_segmented:
        table = tile_starts_for(case.segment_lens)
        starts = torch.tensor(table, dtype=torch.int32)
        tiles = len(table) - 1
    inputs = Inputs(query, key, positions, cache_for(case.flavour), _last_index(case), starts, tiles,
                    int(case.is_segmented))
    return inputs if str(device) == "cpu" else inputs.to(device)


def min_bytes(case: Case) -> int:
    """Algorithmic minimum HBM bytes of one launch (each byte once; cos/sin
    rows once per distinct position)."""
    n, bs = case.n_tokens, case.batch_size
    seg = 4 * (len(tile_starts_for(case.segment_lens))) if case.is_segmented else 0
    if case.is_mirror:
        # K: rope slice read+write (256) + cos/sin row (256) + position (8) per
        # token; Q: 6 slices read+write (1536) + last_index (8) per row.
        return 520 * n + 1544 * bs + seg
    # Q 6 slices + K 1 slice read+write (1792), cos/sin row (256), position (8).
    return 2056 * n + seg
