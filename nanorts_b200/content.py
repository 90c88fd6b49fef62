"""Scenario content: MicroRTS map documents -> GameConfig.

Host-side, runs once per scenario.  Follows the reference's loader:
  document checks       src/nanorts/content/acceptance.py:24-164
  bucket derivation     src/nanorts/content/normalize.py:45-93
  slot claiming         src/nanorts/content/normalize.py:119-170
  capacity profiles     src/nanorts/content/scenarios.py:20-42

The shipped maps are bundled as ``maps/maps.json`` (terrain, players and
units of every MicroRTS map up to 64x64 that NanoRTS ships, converted by
``maps/extract.py``); ``load_game`` also reads any MicroRTS XML map file.
"""

from __future__ import annotations

import dataclasses
import functools
import json
import os
import re
from pathlib import Path
from xml.etree import ElementTree

import numpy as np

from nanorts_b200.model import (
    OWNER_NEUTRAL,
    PLAYER_COUNT,
    TABLES,
    BucketSpec,
    ConflictStrategy,
    GameConfig,
    ModelError,
    UnitType,
    UnitTypeTableVersion,
    content_hash,
    empty_state,
)

MAP_FILE = Path(__file__).resolve().parent / "maps" / "maps.json"

# Profiled per-player slot counts (scenarios.py:20-22).
CAPACITY_PROFILES = {"basesWorkers8x8": 52, "basesWorkers16x16": 70}

_INTEGER = re.compile(r"[+-]?[0-9]+")


class ContentError(ModelError):
    """A map document the loader refuses."""


@dataclasses.dataclass(frozen=True)
class UnitRecord:
    type: str
    id: int
    player: int
    x: int
    y: int
    hitpoints: int
    resources: int


@dataclasses.dataclass(frozen=True)
class ContentDocument:
    width: int
    height: int
    terrain: str
    players: tuple[tuple[int, int], ...]
    units: tuple[UnitRecord, ...]


def _int_attribute(element: ElementTree.Element, name: str) -> int:
    text = element.get(name)
    if text is None or _INTEGER.fullmatch(text) is None:
        raise ContentError(f"<{element.tag}> attribute {name}={text!r} is not an integer")
    return int(text)


def document_from_xml(text: str) -> ContentDocument:
    """Parse a MicroRTS ``rts.PhysicalGameState`` XML document."""
    try:
        root = ElementTree.fromstring(text)
    except ElementTree.ParseError as error:
        raise ContentError(f"the document is not well formed XML: {error}") from error

    def child(name: str) -> ElementTree.Element:
        found = root.find(name)
        if found is None:
            raise ContentError(f"the document has no <{name}> element")
        return found

    players = tuple((_int_attribute(p, "ID"), _int_attribute(p, "resources")) for p in child("players"))
    units = tuple(
        UnitRecord(
            type=u.get("type") or "",
            id=_int_attribute(u, "ID"),
            player=_int_attribute(u, "player"),
            x=_int_attribute(u, "x"),
            y=_int_attribute(u, "y"),
            hitpoints=_int_attribute(u, "hitpoints"),
            resources=_int_attribute(u, "resources"),
        )
        for u in child("units")
    )
    return ContentDocument(
        width=_int_attribute(root, "width"),
        height=_int_attribute(root, "height"),
        terrain=(child("terrain").text or "").strip(),
        players=players,
        units=units,
    )


def _check_document(document: ContentDocument, table: tuple[UnitType, ...]) -> None:
    """The acceptance clauses of ``acceptance.py:137-164``."""
    if document.width <= 0 or document.height <= 0:
        raise ContentError(f"the field is {document.width}x{document.height}, expected positive extents")
    if len(document.terrain) != document.width * document.height or set(document.terrain) - set("01"):
        raise ContentError("the <terrain> payload is not one binary digit per cell")
    if len(document.players) != PLAYER_COUNT or any(d != e for e, (d, _) in enumerate(document.players)):
        raise ContentError(f"expected exactly {PLAYER_COUNT} positional player records")
    names = {unit.name for unit in table}
    seen_ids: set[int] = set()
    occupied: set[tuple[int, int]] = set()
    for unit in document.units:
        if unit.type not in names:
            raise ContentError(f"unit ID {unit.id} names the unknown type {unit.type!r}")
        if unit.id in seen_ids:
            raise ContentError(f"unit ID {unit.id} is declared more than once")
        seen_ids.add(unit.id)
        if not (0 <= unit.x < document.width and 0 <= unit.y < document.height):
            raise ContentError(f"unit ID {unit.id} sits outside the field")
        if (unit.x, unit.y) in occupied:
            raise ContentError(f"unit ID {unit.id} sits on an occupied cell")
        occupied.add((unit.x, unit.y))
        if unit.player != OWNER_NEUTRAL and unit.player not in range(PLAYER_COUNT):
            raise ContentError(f"unit ID {unit.id} names undeclared player {unit.player}")
        if not 0 <= unit.hitpoints < 2**15:
            raise ContentError(f"unit ID {unit.id} declares {unit.hitpoints} hit points")


def _population(document: ContentDocument, owner: int) -> int:
    return sum(1 for unit in document.units if unit.player == owner)


def _resource_bound(document: ContentDocument, table: tuple[UnitType, ...]) -> int | None:
    """Largest population a player can ever field (``normalize.py:45-74``)."""
    produced = [unit for unit in table if unit.produced_by]
    harvesters = [unit for unit in table if unit.can_harvest]
    applies = (
        bool(produced)
        and bool(harvesters)
        and all(unit.cost > 0 and not unit.is_resource for unit in produced)
        and all(not unit.is_resource and unit.harvest_amount >= 0 for unit in harvesters)
    )
    if not applies:
        return None
    types = {unit.name: unit for unit in table}
    largest_harvest = max(unit.harvest_amount for unit in harvesters)
    on_map = sum(
        max(unit.resources, 1) + largest_harvest - 1 if types[unit.type].is_resource else max(unit.resources, 0)
        for unit in document.units
    )
    cheapest = min(unit.cost for unit in produced)
    return max(_population(document, player) + max(0, balance + on_map) // cheapest
               for player, balance in document.players)


def derive_bucket(document: ContentDocument, table: tuple[UnitType, ...], utt: UnitTypeTableVersion,
                  conflict_strategy: ConflictStrategy) -> BucketSpec:
    cells = document.height * document.width
    bound = _resource_bound(document, table)
    return BucketSpec(
        height=document.height,
        width=document.width,
        neutral_capacity=_population(document, OWNER_NEUTRAL),
        per_player_capacity=cells if bound is None else max(1, min(cells, bound)),
        unit_type_capacity=len(table),
        attack_offset_capacity=(2 * max(unit.attack_range for unit in table) + 1) ** 2,
        utt_identity=utt,
        utt_content_hash=content_hash(table),
        conflict_strategy=conflict_strategy,
    )


def _initial_state(document: ContentDocument, table: tuple[UnitType, ...], bucket: BucketSpec) -> dict[str, np.ndarray]:
    """Units claim the next free slot of their block in document order; births are document positions."""
    names = {unit.name: index for index, unit in enumerate(table)}
    state = empty_state(bucket)
    next_free = [0] * (PLAYER_COUNT + 1)
    entity_at = state["entity_at"].reshape(-1)
    for position, unit in enumerate(document.units):
        if unit.player == OWNER_NEUTRAL:
            start, capacity = 0, bucket.neutral_capacity
        else:
            start, capacity = bucket.player_slot_start(unit.player), bucket.per_player_capacity
        offset = next_free[unit.player + 1]
        if offset >= capacity:
            raise ContentError(f"the block of player {unit.player} holds {capacity} slots, which unit ID {unit.id} exceeds")
        next_free[unit.player + 1] = offset + 1
        slot = start + offset
        cell = unit.x + unit.y * bucket.width
        state["birth"][slot] = position
        state["unit_type"][slot] = names[unit.type]
        state["owner"][slot] = unit.player
        state["cell"][slot] = cell
        state["hit_points"][slot] = unit.hitpoints
        state["carried_resources"][slot] = unit.resources
        entity_at[cell] = slot
    state["player_resources"][:] = [resources for _, resources in document.players]
    state["next_birth"][...] = len(document.units)
    return state


def decide(state: dict[str, np.ndarray], bucket: BucketSpec) -> dict[str, np.ndarray]:
    """``outcome.decide`` (core/outcome.py:11-19) on one game's host state."""
    out = dict(state)
    active = state["birth"][bucket.neutral_capacity:] != -1
    surviving = active.reshape(PLAYER_COUNT, bucket.per_player_capacity).any(axis=1)
    count = int(surviving.sum())
    out["game_over"] = np.asarray(count <= 1)
    out["winner"] = np.asarray(int(np.argmax(surviving)) if count == 1 else -1, np.int32)
    return out


def assemble_game(document: ContentDocument, *, utt: UnitTypeTableVersion = UnitTypeTableVersion.ORIGINAL_FINETUNED,
                  conflict_strategy: ConflictStrategy = ConflictStrategy.CANCEL_BOTH, max_cycles: int = 5000,
                  per_player_capacity: int | None = None) -> GameConfig:
    utt = UnitTypeTableVersion(utt)
    conflict_strategy = ConflictStrategy(conflict_strategy)
    table = TABLES[utt]
    _check_document(document, table)
    bucket = derive_bucket(document, table, utt, conflict_strategy)
    if per_player_capacity is not None:
        floor = max(_population(document, p) for p in range(PLAYER_COUNT))
        if not floor <= per_player_capacity <= bucket.cell_count:
            raise ContentError(f"per_player_capacity {per_player_capacity} is outside [{floor}, {bucket.cell_count}]")
        bucket = dataclasses.replace(bucket, per_player_capacity=per_player_capacity)
    if max_cycles <= 0:
        raise ModelError(f"max_cycles is {max_cycles}, expected a positive horizon")
    terrain = np.asarray([c == "1" for c in document.terrain], bool).reshape(bucket.height, bucket.width)
    return GameConfig(terrain=terrain, max_cycles=int(max_cycles), initial_state=_initial_state(document, table, bucket),
                      unit_types=table, bucket=bucket)


def load_game(path: str | os.PathLike[str], **options) -> GameConfig:
    """Load any MicroRTS XML map (``content/loading.py:169-174``)."""
    return assemble_game(document_from_xml(Path(path).read_text(encoding="utf-8")), **options)


@functools.cache
def _bundled() -> dict[str, dict]:
    return json.loads(MAP_FILE.read_text())


def scenario_names() -> tuple[str, ...]:
    return tuple(sorted(_bundled()))


def shipped_document(name: str) -> ContentDocument:
    maps = _bundled()
    if name not in maps:
        raise ModelError(f"map_name_to_scenario refuses scenario {name!r}: it is none of the {len(maps)} bundled maps")
    record = maps[name]
    return ContentDocument(
        width=record["width"],
        height=record["height"],
        terrain=record["terrain"],
        players=tuple(tuple(p) for p in record["players"]),
        units=tuple(UnitRecord(*u) for u in record["units"]),
    )


def map_name_to_scenario(name: str, *, utt: UnitTypeTableVersion = UnitTypeTableVersion.ORIGINAL_FINETUNED,
                         conflict_strategy: ConflictStrategy = ConflictStrategy.CANCEL_BOTH, max_cycles: int = 5000,
                         capacity_profile: bool = True) -> GameConfig:
    """Shipped scenario by name, with the profiled slot count unless ``capacity_profile=False``."""
    document = shipped_document(name)
    game = assemble_game(document, utt=utt, conflict_strategy=conflict_strategy, max_cycles=max_cycles)
    profile = CAPACITY_PROFILES.get(name)
    if profile is None or not capacity_profile or profile >= game.bucket.per_player_capacity:
        return game
    return assemble_game(document, utt=utt, conflict_strategy=conflict_strategy, max_cycles=max_cycles,
                         per_player_capacity=profile)


def with_unit_type_table(game: GameConfig, utt: UnitTypeTableVersion) -> GameConfig:
    """Swap the unit type table of a scenario (``loading.py:189-210``)."""
    utt = UnitTypeTableVersion(utt)
    if utt == game.bucket.utt_identity:
        return game
    table = TABLES[utt]
    if tuple(u.name for u in table) != tuple(u.name for u in game.unit_types):
        raise ContentError(f"unit type table {utt} declares other types than the scenario")
    if (2 * max(u.attack_range for u in table) + 1) ** 2 != game.bucket.attack_offset_capacity:
        raise ContentError(f"unit type table {utt} derives another attack window")
    bucket = dataclasses.replace(game.bucket, utt_identity=utt, utt_content_hash=content_hash(table))
    return dataclasses.replace(game, unit_types=table, bucket=bucket)
