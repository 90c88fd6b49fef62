"""Small hand-built scenarios and Commands for the rule known-answer tests."""

from __future__ import annotations

import numpy as np

from nanorts_b200.content import ContentDocument, UnitRecord, assemble_game
from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion

KIND = {"none": 0, "move": 1, "harvest": 2, "return": 3, "produce": 4, "attack": 5}
UP, RIGHT, DOWN, LEFT = 0, 1, 2, 3


def tiny_game(units, *, width=4, height=4, resources=(5, 5), walls=(), strategy=ConflictStrategy.CANCEL_BOTH,
              max_cycles=5000, utt=UnitTypeTableVersion.ORIGINAL):
    """units: (type, player, x, y, hitpoints, resources) in document order."""
    terrain = ["0"] * (width * height)
    for x, y in walls:
        terrain[y * width + x] = "1"
    document = ContentDocument(
        width=width, height=height, terrain="".join(terrain),
        players=((0, resources[0]), (1, resources[1])),
        units=tuple(UnitRecord(t, i, p, x, y, hp, r) for i, (t, p, x, y, hp, r) in enumerate(units)),
    )
    return assemble_game(document, utt=utt, conflict_strategy=strategy, max_cycles=max_cycles)


class CommandSheet:
    """Commands int32[1, 6, 2, C] for one game: (kind, direction, none_duration,
    target_cell, produced_type, request_order) per player slot."""

    def __init__(self, game):
        self.C = game.bucket.per_player_capacity
        self.array = np.full((1, 6, 2, self.C), -1, np.int32)
        self.array[0, 2] = 0  # none_duration

    def set(self, player, local, kind, *, direction=-1, none_duration=None, target=-1, produced=-1):
        a = self.array[0]
        a[0, player, local] = KIND[kind]
        a[1, player, local] = direction
        a[2, player, local] = (1 if kind == "none" else 0) if none_duration is None else none_duration
        a[3, player, local] = target
        a[4, player, local] = produced
        return self


def idle(game):
    return CommandSheet(game).array


def state_invariants(state: dict, bucket) -> list[str]:
    """The reference's state invariants (model/state.py:87-165) over every lane."""
    problems = []
    E, cells = bucket.entity_capacity, bucket.cell_count
    N, C = bucket.neutral_capacity, bucket.per_player_capacity
    fills = {"birth": -1, "unit_type": -1, "owner": -1, "cell": -1, "hit_points": 0, "carried_resources": 0,
             "pending_kind": -1, "pending_direction": -1, "pending_none_duration": 0, "pending_target_cell": -1,
             "pending_produced_type": -1, "pending_issued_at": 0, "pending_completes_at": 0, "pending_order": -1}
    block_owner = np.concatenate([np.full(N, -1), np.zeros(C), np.ones(C)]).astype(np.int64)
    for lane in range(state["birth"].shape[0]):
        active = state["birth"][lane] != -1
        cell = state["cell"][lane].astype(np.int64)
        entity_at = state["entity_at"][lane].reshape(-1).astype(np.int64)
        if np.any(active & ((cell < 0) | (cell >= cells))):
            problems.append(f"lane {lane}: active cell off the field")
        for s in np.flatnonzero(active):
            if entity_at[cell[s]] != s:
                problems.append(f"lane {lane}: slot {s} missing from entity_at")
        for c in np.flatnonzero(entity_at != -1):
            s = entity_at[c]
            if not (0 <= s < E and active[s] and cell[s] == c):
                problems.append(f"lane {lane}: entity_at[{c}] names slot {s} that is not there")
        if np.any(active & (state["owner"][lane].astype(np.int64) != block_owner)):
            problems.append(f"lane {lane}: owner disagrees with the slot block")
        for name, fill in fills.items():
            if np.any(~active & (state[name][lane] != fill)):
                problems.append(f"lane {lane}: {name} not canonical on an inactive slot")
    return problems
