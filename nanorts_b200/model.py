"""Game model: vocabulary, unit type tables, bucket extents and the State layout.

The layouts here are the drop-in contract with NanoRTS: every State leaf has
the name, per-game shape, dtype and canonical-empty fill of the reference's
``State`` pytree (``src/nanorts/model/state.py:27-84``), so a batch of games is
one lane-major array per leaf, ``[L, *shape]``, exactly as ``jax.vmap`` lays
the reference's state out.

Reference anchors:
  vocabulary          src/nanorts/model/vocabulary.py:1-53
  unit types/tables   src/nanorts/model/unit_types.py:16-148
  bucket extents      src/nanorts/model/bucket.py:24-105
  index dtypes        src/nanorts/model/leaf.py:85-98
"""

from __future__ import annotations

import dataclasses
import enum
import hashlib
import json
import math
from typing import Final

import numpy as np

ABSENT: Final = -1
OWNER_NEUTRAL: Final = -1
PLAYER_COUNT: Final = 2
ATTACK_TARGET_OWNER_COUNT: Final = 3

KIND_ABSENT: Final = -1
KIND_NONE: Final = 0
KIND_MOVE: Final = 1
KIND_HARVEST: Final = 2
KIND_RETURN: Final = 3
KIND_PRODUCE: Final = 4
KIND_ATTACK: Final = 5
ACTION_KIND_COUNT: Final = 6

DIRECTION_UP: Final = 0
DIRECTION_RIGHT: Final = 1
DIRECTION_DOWN: Final = 2
DIRECTION_LEFT: Final = 3
DIRECTION_COUNT: Final = 4
DIRECTION_OFFSETS: Final = ((0, -1), (1, 0), (0, 1), (-1, 0))


class ModelError(ValueError):
    """Raised for a configuration or value the model refuses."""


class UnitTypeTableVersion(enum.StrEnum):
    ORIGINAL = "VERSION_ORIGINAL"
    ORIGINAL_FINETUNED = "VERSION_ORIGINAL_FINETUNED"


class ConflictStrategy(enum.StrEnum):
    CANCEL_BOTH = "CANCEL_BOTH"
    CANCEL_RANDOM = "CANCEL_RANDOM"
    CANCEL_ALTERNATING = "CANCEL_ALTERNATING"


STRATEGY_CODES: Final = {
    ConflictStrategy.CANCEL_BOTH: 0,
    ConflictStrategy.CANCEL_RANDOM: 1,
    ConflictStrategy.CANCEL_ALTERNATING: 2,
}


@dataclasses.dataclass(frozen=True)
class UnitType:
    """One row of a unit type table (MicroRTS ``UnitType``)."""

    name: str
    cost: int = 1
    hit_points: int = 1
    produce_time: int = 10
    move_time: int = 10
    attack_time: int = 10
    harvest_time: int = 10
    attack_range: int = 1
    attack_damage: int = 1
    harvest_amount: int = 1
    sight_radius: int = 4
    is_resource: bool = False
    is_stockpile: bool = False
    can_harvest: bool = False
    can_move: bool = True
    can_attack: bool = True
    produced_by: tuple[str, ...] = ()


_RESOURCE = UnitType("Resource", sight_radius=0, is_resource=True, can_move=False, can_attack=False)
_BASE = UnitType("Base", cost=10, hit_points=10, produce_time=250, sight_radius=5, is_stockpile=True,
                 can_move=False, can_attack=False, produced_by=("Worker",))
_BARRACKS = UnitType("Barracks", cost=5, hit_points=4, produce_time=200, sight_radius=3, can_move=False,
                     can_attack=False, produced_by=("Worker",))
_WORKER = UnitType("Worker", produce_time=50, attack_time=5, harvest_time=20, sight_radius=3,
                   can_harvest=True, produced_by=("Base",))
_LIGHT = UnitType("Light", cost=2, hit_points=4, produce_time=80, move_time=8, attack_time=5,
                  attack_damage=2, sight_radius=2, produced_by=("Barracks",))
_HEAVY = UnitType("Heavy", cost=2, hit_points=4, produce_time=120, move_time=12, attack_time=5,
                  attack_damage=4, sight_radius=2, produced_by=("Barracks",))
_RANGED = UnitType("Ranged", cost=2, produce_time=100, attack_time=5, attack_range=3, sight_radius=3,
                   produced_by=("Barracks",))

TYPE_RESOURCE, TYPE_BASE, TYPE_BARRACKS, TYPE_WORKER, TYPE_LIGHT, TYPE_HEAVY, TYPE_RANGED = range(7)

TABLES: Final = {
    UnitTypeTableVersion.ORIGINAL: (_RESOURCE, _BASE, _BARRACKS, _WORKER, _LIGHT, _HEAVY, _RANGED),
    # The competition table differs in five values (unit_types.py:131-139).
    UnitTypeTableVersion.ORIGINAL_FINETUNED: (
        _RESOURCE,
        dataclasses.replace(_BASE, produce_time=200),
        dataclasses.replace(_BARRACKS, produce_time=100),
        _WORKER,
        _LIGHT,
        dataclasses.replace(_HEAVY, cost=3, hit_points=8, move_time=10),
        _RANGED,
    ),
}

# Column order of the packed unit table handed to the kernels and the oracle.
UNIT_COLUMNS: Final = (
    "cost", "hit_points", "produce_time", "move_time", "attack_time", "harvest_time", "attack_range",
    "attack_damage", "harvest_amount", "sight_radius", "is_resource", "is_stockpile", "can_harvest",
    "can_move", "can_attack",
)
UNIT_COLUMN_COUNT: Final = len(UNIT_COLUMNS)  # followed by one "produces" column per type


def unit_table(table: tuple[UnitType, ...]) -> np.ndarray:
    """``int32[T, 15 + T]``: the scalar columns, then ``produces[producer, produced]``.

    ``produces`` follows ``unit_types.py:115-121``: a type produces another when its
    name is in the other's ``produced_by``.
    """
    names = [unit.name for unit in table]
    if len(set(names)) != len(names):
        raise ModelError(f"the table declares a type more than once: {names}")
    rows = []
    for producer in table:
        row = [int(getattr(producer, column)) for column in UNIT_COLUMNS]
        row += [int(producer.name in produced.produced_by) for produced in table]
        rows.append(row)
    return np.asarray(rows, np.int32)


def content_hash(table: tuple[UnitType, ...]) -> str:
    payload = unit_table(table).tolist()
    return hashlib.sha256(json.dumps(payload, separators=(",", ":")).encode()).hexdigest()


@dataclasses.dataclass(frozen=True)
class BucketSpec:
    """Static extents of one scenario (``bucket.py:24-105``)."""

    height: int
    width: int
    neutral_capacity: int
    per_player_capacity: int
    unit_type_capacity: int
    attack_offset_capacity: int
    utt_identity: UnitTypeTableVersion
    utt_content_hash: str
    conflict_strategy: ConflictStrategy

    @property
    def cell_count(self) -> int:
        return self.height * self.width

    @property
    def entity_capacity(self) -> int:
        return self.neutral_capacity + PLAYER_COUNT * self.per_player_capacity

    @property
    def attack_window_side(self) -> int:
        return math.isqrt(self.attack_offset_capacity)

    @property
    def max_attack_range(self) -> int:
        return (self.attack_window_side - 1) // 2

    def player_slot_start(self, player: int) -> int:
        return self.neutral_capacity + player * self.per_player_capacity

    @property
    def index_dtype(self) -> np.dtype:
        """CELL_INDEX/SLOT_INDEX dtype: int16 while both extents fit (``leaf.py:85-98``)."""
        widest = max(self.cell_count, self.entity_capacity)
        return np.dtype(np.int16) if widest <= np.iinfo(np.int16).max else np.dtype(np.int32)

    @property
    def mask_width(self) -> int:
        return ACTION_KIND_COUNT + 4 * DIRECTION_COUNT + self.unit_type_capacity + self.attack_offset_capacity


# State leaves in the reference's declaration order (state.py:35-80), with the
# per-game shape class, dtype and canonical-empty fill.  "index" is the bucket's
# CELL_INDEX / SLOT_INDEX dtype.
SLOT_LEAVES: Final = (
    ("birth", "int32", ABSENT),
    ("unit_type", "int8", ABSENT),
    ("owner", "int8", ABSENT),
    ("cell", "index", ABSENT),
    ("hit_points", "int16", 0),
    ("carried_resources", "int32", 0),
    ("pending_kind", "int8", KIND_ABSENT),
    ("pending_direction", "int8", ABSENT),
    ("pending_none_duration", "int32", 0),
    ("pending_target_cell", "index", ABSENT),
    ("pending_produced_type", "int8", ABSENT),
    ("pending_issued_at", "int32", 0),
    ("pending_completes_at", "int32", 0),
    ("pending_order", "int32", ABSENT),
)
FIELD_LEAVES: Final = (("entity_at", "index", ABSENT),)
SCALAR_LEAVES: Final = (
    ("time", "int32", (), 0),
    ("player_resources", "int32", (PLAYER_COUNT,), 0),
    ("next_birth", "int32", (), 0),
    ("next_pending_order", "int32", (), 0),
    ("alternating_conflict_count", "int32", (), 0),
    ("game_over", "bool", (), False),
    ("winner", "int32", (), ABSENT),
    ("spawn_overflow", "int32", (PLAYER_COUNT,), 0),  # State.telemetry.spawn_overflow
)


def leaf_dtype(name: str, bucket: BucketSpec) -> np.dtype:
    return bucket.index_dtype if name == "index" else np.dtype(name)


def leaf_shapes(bucket: BucketSpec) -> dict[str, tuple[tuple[int, ...], np.dtype, object]]:
    """``{leaf: (per-game shape, dtype, fill)}`` in declaration order."""
    shapes: dict[str, tuple[tuple[int, ...], np.dtype, object]] = {}
    for name, dtype, fill in SLOT_LEAVES:
        shapes[name] = ((bucket.entity_capacity,), leaf_dtype(dtype, bucket), fill)
    for name, dtype, fill in FIELD_LEAVES:
        shapes[name] = ((bucket.height, bucket.width), leaf_dtype(dtype, bucket), fill)
    for name, dtype, shape, fill in SCALAR_LEAVES:
        shapes[name] = (shape, np.dtype(dtype), fill)
    return shapes


def empty_state(bucket: BucketSpec) -> dict[str, np.ndarray]:
    """The canonical empty State of one game (``leaf.py:205-240``)."""
    return {name: np.full(shape, fill, dtype) for name, (shape, dtype, fill) in leaf_shapes(bucket).items()}


@dataclasses.dataclass(frozen=True, eq=False)
class GameConfig:
    """A scenario: terrain, horizon, initial State, unit table and extents (``config.py:209-253``)."""

    terrain: np.ndarray  # bool[H, W]
    max_cycles: int
    initial_state: dict[str, np.ndarray]
    unit_types: tuple[UnitType, ...]
    bucket: BucketSpec

    @property
    def table(self) -> np.ndarray:
        return unit_table(self.unit_types)

    def column(self, name: str) -> np.ndarray:
        return self.table[:, UNIT_COLUMNS.index(name)]
