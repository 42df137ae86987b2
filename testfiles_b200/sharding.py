"""Request sharding for data-parallel RoPE over several GPUs.

Tokens and requests are independent, so a batch is split across ranks with
no exchange on the hot path; each rank runs the same single-GPU op on its
shard.  Collectives are used only after the op, to bring results back for
checking (:func:`gather_rows`).

* Ordinary single request: contiguous, 64-aligned token ranges
  (:func:`shard_tokens`).
* Segmented / mirror batches: whole requests, contiguous in request order,
  balanced by token count (:func:`shard_requests`); each rank gets its K rows,
  its Q rows, ``last_index`` rebased to its local token offset and a locally
  rebuilt ``segment_tile_starts`` (:func:`local_batch`).

Failures stay on the host: each rank folds its C-ABI return code and device
status word into one integer, and :func:`agree_status` (a MAX all-reduce,
the step before any gather) tells every rank whether any rank failed, so all
ranks take the same next collective or none.  A rank that died outright
surfaces as an error of that collective within the process group's timeout.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch

TILE_TOKENS = 64


def shard_tokens(n_tokens: int, world_size: int, rank: int, align: int = TILE_TOKENS) -> tuple[int, int]:
    """[begin, end) of ``rank``'s token range: 64-aligned chunks, as even as possible."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("bad rank / world_size")
    chunks = (n_tokens + align - 1) // align
    base, extra = divmod(chunks, world_size)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return min(first * align, n_tokens), min((first + count) * align, n_tokens)


def shard_requests(segment_lens: Sequence[int], world_size: int) -> list[tuple[int, int]]:
    """Contiguous request ranges [r0, r1) per rank, balanced by tokens.

    Rank ``i`` takes the requests whose token midpoint falls in
    ``[i * N / W, (i + 1) * N / W)``; every request goes to exactly one rank.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    total = sum(int(x) for x in segment_lens)
    bounds = [0] * (world_size + 1)
    bounds[world_size] = len(segment_lens)
    token = 0
    rank = 0
    for r, length in enumerate(segment_lens):
        mid2 = 2 * token + int(length)  # twice the request's token midpoint
        while rank < world_size - 1 and mid2 * world_size >= 2 * total * (rank + 1):
            rank += 1
            bounds[rank] = r
        token += int(length)
    for i in range(rank + 1, world_size):
        bounds[i] = len(segment_lens)
    return [(bounds[i], bounds[i + 1]) for i in range(world_size)]


@dataclass
class LocalBatch:
    """One rank's view of a segmented batch."""

    request_begin: int
    request_end: int
    token_begin: int
    token_end: int
    segment_lens: tuple[int, ...]
    last_index: list[int]            # rebased to the local token offset
    tile_starts: list[int]           # rebuilt locally, [T_local + 1]

    @property
    def n_tokens(self) -> int:
        return self.token_end - self.token_begin

    @property
    def num_work_tiles(self) -> int:
        return len(self.tile_starts) - 1


def local_batch(segment_lens: Sequence[int], request_range: tuple[int, int],
                last_index: Optional[Sequence[int]] = None) -> LocalBatch:
    """Slice requests [r0, r1): token range, rebased last_index, local tiles.

    ``last_index`` defaults to each request's last token; a given one is
    rebased by the rank's token offset (it must point inside the rank's
    requests).
    """
    r0, r1 = request_range
    lens = tuple(int(x) for x in segment_lens)
    token_begin = sum(lens[:r0])
    local = lens[r0:r1]
    token_end = token_begin + sum(local)
    if last_index is None:
        rebased, end = [], 0
        for length in local:
            end += length
            rebased.append(end - 1)
    else:
        rebased = [int(v) - token_begin for v in list(last_index)[r0:r1]]
        if any(v < 0 or v >= token_end - token_begin for v in rebased):
            raise ValueError("last_index points outside the rank's requests")
    starts: list[int] = []
    token = 0
    for length in local:
        starts.extend(range(token, token + length, TILE_TOKENS))
        token += length
    starts.append(token)
    return LocalBatch(r0, r1, token_begin, token_end, local, rebased, starts)


def gather_rows(local: torch.Tensor, counts: Sequence[int], group=None) -> Optional[torch.Tensor]:
    """Gather variable-length row blocks to rank 0 (None elsewhere).

    Rows are padded to ``max(counts)`` so one ``all_gather_into_tensor`` (or
    ``all_gather`` on backends without it) moves everything; rank 0 strips the
    padding and concatenates in rank order.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    width = max(int(c) for c in counts) if counts else 0
    padded = torch.zeros((width, *local.shape[1:]), dtype=local.dtype, device=local.device)
    if local.shape[0]:
        padded[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * width, *local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, padded, group=group)
        parts = list(out.split(width)) if width else [out[:0]] * world
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
    if rank != 0:
        return None
    return torch.cat([p[: int(c)] for p, c in zip(parts, counts)], dim=0)


class RankFailure(RuntimeError):
    """Raised on every rank when any rank reported a non-zero status."""

    def __init__(self, status: int):
        super().__init__(f"a rank reported status {status:#x}; the gather was skipped on every rank")
        self.status = status


def agree_status(status: int, group=None, device: Optional[torch.device] = None) -> int:
    """MAX of every rank's status; every rank gets the same answer.

    ``status`` is 0 for success.  Fold a C-ABI return code ``rc`` and a device
    status word ``dev`` as ``rc << 8 | dev`` so either one makes it non-zero.
    NCCL groups need ``device`` (the rank's CUDA device); gloo runs on CPU.
    """
    import torch.distributed as dist

    if status < 0:
        raise ValueError("status must be non-negative")
    if device is None:
        device = torch.device("cpu")
    t = torch.tensor([int(status)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return int(t.item())


def check_all_ranks(status: int, group=None, device: Optional[torch.device] = None) -> None:
    """:func:`agree_status`, raising :class:`RankFailure` on every rank if any failed."""
    agreed = agree_status(status, group, device)
    if agreed:
        raise RankFailure(agreed)
