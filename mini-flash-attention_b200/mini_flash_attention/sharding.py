"""Multi-GPU partition of the attention forward (one process per GPU, no collective).

Every (batch*head) row of the [B*H, N, D] problem is independent, so the path shards by
contiguous blocks of batch*head rows: rank r owns rows [start, stop) of q, k, v and out, which
are contiguous slices of memory. With fewer batch*head rows than ranks, every query row is
still independent once a rank holds the whole k and v: the ranks then split the query rows of
every head instead (`q_shard`, computed by `forward_rows`). Nothing crosses GPUs on the hot
path; a caller that wants the whole output back gathers the slices outside the timed region.

The reference has no multi-GPU mode; this module only decides who owns what.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int  # first batch*head row owned by this rank
    stop: int   # one past the last

    @property
    def rows(self) -> int:
        return self.stop - self.start


def bh_shard(total_bh: int, rank: int, world: int) -> Shard:
    """Contiguous, balanced split of `total_bh` rows over `world` ranks (sizes differ by <= 1,
    the first total_bh % world ranks take one extra row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    if total_bh < 0:
        raise ValueError("negative batch*head")
    base, extra = divmod(total_bh, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return Shard(rank, world, start, stop)


def all_shards(total_bh: int, world: int) -> list[Shard]:
    return [bh_shard(total_bh, r, world) for r in range(world)]


# query rows of one forward unit (two 128-row tiles): range boundaries on these keep every
# unit whole on one rank
Q_ALIGN = 256


@dataclass(frozen=True)
class QShard:
    rank: int
    world: int
    begin: int  # first query row (of every head) computed by this rank
    end: int    # one past the last

    @property
    def rows(self) -> int:
        return self.end - self.begin


def q_shard(n: int, rank: int, world: int, align: int = Q_ALIGN,
            causal: bool = False) -> QShard:
    """Contiguous split of the query rows [0, n) over `world` ranks in blocks of `align` rows
    (the last block may be short; ranks past the number of blocks get an empty range at n).
    Without the mask every row costs the same: block counts differ by <= 1, the first ranks
    take the extra blocks. With it row i attends to i + 1 keys, so rows [0, x) cost about x^2:
    rank r ends at block round(blocks * sqrt((r + 1) / world))."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    if n < 0 or align <= 0:
        raise ValueError("negative sequence length or bad alignment")
    blocks = -(-n // align)
    if causal:
        def edge(r: int) -> int:
            return round(blocks * math.sqrt(r / world))
        b0, b1 = edge(rank), edge(rank + 1)
    else:
        base, extra = divmod(blocks, world)
        b0 = rank * base + min(rank, extra)
        b1 = b0 + base + (1 if rank < extra else 0)
    return QShard(rank, world, min(b0 * align, n), min(b1 * align, n))


def shard_mode(total_bh: int, world: int) -> str:
    """'rows': batch*head rows per rank (bh_shard); 'queries': query rows of every head per rank
    (q_shard, the whole k and v on every rank), when there are fewer batch*head rows than ranks."""
    return "rows" if total_bh >= world else "queries"
