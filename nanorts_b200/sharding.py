"""Data-parallel sharding of a batch of games over the GPUs of one box.

Games are independent, so a batch of G games splits into contiguous blocks,
one per rank (the leading lane axis of every leaf, as
``NamedSharding(Mesh(devices, ('env',)), P('env'))`` would place the
reference's vmapped state).  Nothing is exchanged while stepping; one
all-reduce of a few integer episode statistics runs at the end.
"""

from __future__ import annotations

import dataclasses

import torch

STAT_FIELDS = ("steps", "episodes", "wins_p0", "wins_p1", "draws", "spawn_overflows")


@dataclasses.dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    global_lanes: int

    @property
    def lanes(self) -> int:
        base, extra = divmod(self.global_lanes, self.world)
        return base + (1 if self.rank < extra else 0)

    @property
    def first(self) -> int:
        base, extra = divmod(self.global_lanes, self.world)
        return self.rank * base + min(self.rank, extra)

    def slice(self) -> slice:
        return slice(self.first, self.first + self.lanes)


def shard_keys(keys: torch.Tensor, shard: Shard) -> torch.Tensor:
    """This rank's block of the [G, 2] per-game reset keys."""
    if keys.shape[0] != shard.global_lanes:
        raise ValueError(f"{keys.shape[0]} keys for {shard.global_lanes} games")
    return keys[shard.slice()].contiguous()


class EpisodeStats:
    """Running sums of episode statistics on this rank's device."""

    def __init__(self, device: torch.device | str) -> None:
        self.values = torch.zeros(len(STAT_FIELDS), dtype=torch.int64, device=device)

    def add_step(self, done: torch.Tensor, winner: torch.Tensor, spawn_overflow: torch.Tensor) -> None:
        """One step's outputs of this rank's games (done bool[L], winner int32[L], overflow int32[L, 2])."""
        done = done.to(torch.bool)
        won0 = done & (winner == 0)
        won1 = done & (winner == 1)
        update = torch.stack([
            torch.tensor(done.numel(), device=done.device, dtype=torch.int64),
            done.sum(), won0.sum(), won1.sum(), (done & (winner < 0)).sum(),
            (done & (spawn_overflow > 0).any(dim=-1)).sum(),
        ]).to(self.values.device, torch.int64)
        self.values += update

    def reduce(self, group=None) -> dict[str, int]:
        """Sums over ranks (one all-reduce) when a process group is up."""
        values = self.values.clone()
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(values, op=torch.distributed.ReduceOp.SUM, group=group)
        return dict(zip(STAT_FIELDS, (int(v) for v in values.tolist()), strict=True))
