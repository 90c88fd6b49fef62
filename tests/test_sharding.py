"""Sharding across ranks on CPU: 2 gloo ranks, each stepping its block of
games with the oracle, reduce to the same episode statistics as one process
stepping the whole batch."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanorts_b200.sharding import EpisodeStats, Shard, shard_keys

GAMES, STEPS = 10, 60


def test_shard_blocks_cover_the_batch():
    for world in (1, 2, 3, 4, 8):
        shards = [Shard(r, world, 1003) for r in range(world)]
        assert sum(s.lanes for s in shards) == 1003
        assert [s.first for s in shards] == [sum(t.lanes for t in shards[:r]) for r in range(world)]


def _run(keys: np.ndarray, steps: int) -> torch.Tensor:
    from oracle.oracle import Oracle
    from tests.parity import CONFIGS, sample

    game = CONFIGS["c1_8x8_both"].game(25)
    orc = Oracle(game, keys.shape[0], threads=1)
    orc.reset(keys)
    stats = EpisodeStats("cpu")
    for t in range(steps):
        # actions depend only on the game's own key and step, so any sharding draws the same
        actions = np.stack([sample(orc.legal_masks()[i:i + 1], np.random.default_rng([int(keys[i, 0]), t]))[0]
                            for i in range(keys.shape[0])])
        out = orc.step(actions)
        stats.add_step(torch.from_numpy(out["done"]), torch.from_numpy(out["winner"]),
                       torch.from_numpy(out["spawn_overflow"]))
    return stats.values


def _rank(rank: int, world: int, port: int, keys: np.ndarray, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = Shard(rank, world, keys.shape[0])
        local = shard_keys(torch.from_numpy(keys.view(np.int32)), shard).numpy().view(np.uint32)
        stats = EpisodeStats("cpu")
        stats.values += _run(local, STEPS)
        queue.put((rank, stats.reduce()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_to_the_single_process_statistics():
    keys = np.random.default_rng(3).integers(0, 2**32, size=(GAMES, 2), dtype=np.uint64).astype(np.uint32)
    whole = dict(zip(("steps", "episodes", "wins_p0", "wins_p1", "draws", "spawn_overflows"),
                     _run(keys, STEPS).tolist(), strict=True))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, keys, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1] == whole
    assert whole["steps"] == GAMES * STEPS and whole["episodes"] > 0
