"""Multi-GPU partition of the attention forward (one process per GPU, no collective).

Every (batch*head) row of the [B*H, N, D] problem is independent, so the path shards by
contiguous blocks of batch*head rows: rank r owns rows [start, stop) of q, k, v and out, which
are contiguous slices of memory. Nothing crosses GPUs on the hot path; a caller that wants the
whole output back gathers the slices outside the timed region.

The reference has no multi-GPU mode; this module only decides who owns what.
"""
from __future__ import annotations

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
