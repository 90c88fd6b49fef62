"""Scenario loading: the bundled maps reproduce the reference's extents and
initial states (content/normalize.py:45-170, content/scenarios.py:20-42)."""

from __future__ import annotations

import numpy as np
import pytest

from nanorts_b200 import content, map_name_to_scenario, scenario_names
from nanorts_b200.model import ConflictStrategy, ModelError, UnitTypeTableVersion



@pytest.mark.parametrize("name,kw,neutral,capacity,cells", [
    ("basesWorkers8x8", {}, 2, 47, 64),
    ("basesWorkers16x16", {}, 4, 70, 256),
    ("basesWorkers16x16", {"capacity_profile": False}, 4, 107, 256),
    ("GardenOfWar64x64", {"capacity_profile": False}, 22, 388, 4096),
])
def test_bucket_extents(name, kw, neutral, capacity, cells):
    game = map_name_to_scenario(name, utt=UnitTypeTableVersion.ORIGINAL, **kw)
    b = game.bucket
    assert (b.neutral_capacity, b.per_player_capacity, b.cell_count) == (neutral, capacity, cells)
    assert b.entity_capacity == neutral + 2 * capacity
    assert b.attack_offset_capacity == 49 and b.mask_width == 78 and b.index_dtype == np.int16


def test_initial_state_of_bases8x8():
    game = map_name_to_scenario("basesWorkers8x8")
    s, N, C = game.initial_state, 2, 47
    assert list(s["birth"][:N]) == [0, 1] and list(s["unit_type"][:N]) == [0, 0]
    assert list(s["carried_resources"][:N]) == [20, 20]
    assert list(s["birth"][N:N + 2]) == [2, 4] and list(s["unit_type"][N:N + 2]) == [1, 3]  # p0 base, worker
    assert list(s["birth"][N + C:N + C + 2]) == [3, 5]
    assert s["entity_at"][1, 2] == N and s["entity_at"][1, 1] == N + 1
    assert int(s["next_birth"]) == 6 and list(s["player_resources"]) == [5, 5]


def test_finetuned_table_differs_in_five_values():
    o = map_name_to_scenario("basesWorkers8x8", utt=UnitTypeTableVersion.ORIGINAL).table
    f = map_name_to_scenario("basesWorkers8x8", utt=UnitTypeTableVersion.ORIGINAL_FINETUNED).table
    assert int((o != f).sum()) == 5


def test_unknown_scenario_is_refused():
    with pytest.raises(ModelError):
        map_name_to_scenario("noSuchMap")


def test_bundled_maps_match_the_reference_xml():
    from oracle.oracle import reference_root

    root = reference_root()
    if root is None:
        pytest.skip("no NanoRTS checkout (NANORTS_REFERENCE) to read the map XMLs from")
    reference_maps = root / "src" / "nanorts" / "maps"
    for name in ("basesWorkers8x8", "basesWorkers16x16", "GardenOfWar64x64", "melee4x4light2"):
        path = next(reference_maps.rglob(f"{name}.xml"))
        a = content.load_game(path, utt=UnitTypeTableVersion.ORIGINAL, conflict_strategy=ConflictStrategy.CANCEL_RANDOM)
        b = content.map_name_to_scenario(name, utt=UnitTypeTableVersion.ORIGINAL,
                                         conflict_strategy=ConflictStrategy.CANCEL_RANDOM, capacity_profile=False)
        assert a.bucket == b.bucket
        assert np.array_equal(a.terrain, b.terrain)
        for leaf, value in a.initial_state.items():
            assert np.array_equal(value, b.initial_state[leaf]), leaf
    assert len(scenario_names()) >= 90
