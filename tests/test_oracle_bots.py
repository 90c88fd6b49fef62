"""Known answers for the rush-bot oracle (CPU).

Each case is derived by hand from the reference's source text: the A* pop
order (pathfinding.py:166-228: least f, then the most recently inserted
cell), the building-site ring order (abstraction.py:221-253), the nearest-unit
tie-break by birth (rush.py:31-46) and the script's puts and settling
(rush.py:225-246, abstraction.py:170-219, :1099-1119).
"""

from __future__ import annotations

import numpy as np

from tests.helpers import state_invariants, tiny_game

UP, RIGHT, DOWN, LEFT = 0, 1, 2, 3
MOVE = 1
ABS_ATTACK, ABS_BUILD = 1, 4
TYPE_BASE = 1


def test_astar_straight_line(oracle_lib):
    free = np.ones((5, 5), np.uint8)
    assert oracle_lib.astar(free, 0, 4, 0) == (True, RIGHT, 4, 5)


def test_astar_prefers_the_latest_inserted_of_equal_f(oracle_lib):
    # From (0,0) to (2,2) on an open 3x3: RIGHT and DOWN both have f = 4;
    # DOWN is inserted second and popped first, so the path leaves downwards.
    free = np.ones((3, 3), np.uint8)
    free[0, 0] = 0  # the start cell is occupied by the unit itself
    assert oracle_lib.astar(free, 0, 8, 0) == (True, DOWN, 4, 5)


def test_astar_start_in_range_and_unreachable(oracle_lib):
    free = np.ones((4, 4), np.uint8)
    found, step, distance, pops = oracle_lib.astar(free, 5, 6, 1)
    assert (found, step, distance, pops) == (True, -1, 0, 1)
    walled = np.ones((4, 4), np.uint8)
    walled[:, 2] = 0  # a wall column between start and target
    found, step, distance, pops = oracle_lib.astar(walled, 0, 3, 0)
    assert (found, step, distance) == (False, -1, -1)
    assert pops == 8  # every reachable cell of the left half was popped


def test_astar_detours_around_a_wall(oracle_lib):
    # 3x3, target (2,0), the middle column blocked except its bottom cell.
    free = np.ones((3, 3), np.uint8)
    free[0, 1] = free[1, 1] = 0
    found, step, distance, _ = oracle_lib.astar(free, 0, 2, 0)
    assert (found, step, distance) == (True, DOWN, 6)


def test_worker_rush_builds_a_base_at_the_first_ring_cell(oracle_lib):
    # A lone worker with enough for a base: it is the builder, the site is the
    # top-left corner of ring 1 around it (cell 6 of a 5x5 board), and the
    # walk's search to within 1 of the site steps LEFT (LEFT is inserted after
    # UP with the same f and is popped first).
    game = tiny_game([("Worker", 0, 2, 2, 1, 0), ("Worker", 1, 4, 4, 1, 0)], width=5, height=5, resources=(10, 10))
    orc = oracle_lib.Oracle(game, 1)
    orc.reset(np.zeros((1, 2), np.uint32))
    C = game.bucket.per_player_capacity
    carry = oracle_lib.empty_carry(1, C)
    commands = orc.bot_act(0, oracle_lib.WORKER_RUSH, -1, carry)
    assert commands[0, :, 0, 0].tolist() == [MOVE, LEFT, 0, -1, -1, 0]
    assert (commands[0, 0, 0, 1:] == -1).all() and (commands[0, :, 1] == [[-1], [-1], [0], [-1], [-1], [-1]]).all()
    assert carry["kind"][0, 0] == ABS_BUILD and carry["cell"][0, 0] == 6 and carry["unit_type"][0, 0] == TYPE_BASE
    assert carry["order"][0, 0] == 0 and carry["next_order"][0] == 1 and carry["unit_birth"][0, 0] == 0


def test_melee_attacks_the_nearest_enemy_of_least_birth(oracle_lib):
    # A light unit between two enemy workers at equal distance attacks the one
    # born first (slot order of the document), walking RIGHT toward it.
    game = tiny_game([("Light", 0, 2, 2, 4, 0), ("Worker", 1, 4, 2, 1, 0), ("Worker", 1, 0, 2, 1, 0)],
                     width=5, height=5, resources=(0, 0))
    orc = oracle_lib.Oracle(game, 1)
    orc.reset(np.zeros((1, 2), np.uint32))
    C = game.bucket.per_player_capacity
    carry = oracle_lib.empty_carry(1, C)
    commands = orc.bot_act(0, oracle_lib.WORKER_RUSH, -1, carry)
    target_slot = carry["target"][0, 0]
    assert carry["kind"][0, 0] == ABS_ATTACK
    assert orc.state["cell"][0, target_slot] == 2 * 5 + 4
    assert carry["target_birth"][0, 0] == orc.state["birth"][0, target_slot]
    assert commands[0, 0, 0, 0] == MOVE and commands[0, 1, 0, 0] == RIGHT


def test_idle_units_wait_ten_cycles(oracle_lib):
    # A base with no resources and a lone worker with nothing to harvest or
    # attack: the base gets the filler NONE with the 10-cycle wait, ranked
    # after the kept desires.
    game = tiny_game([("Base", 0, 0, 0, 10, 0), ("Worker", 1, 4, 4, 1, 0)], width=5, height=5, resources=(0, 0))
    orc = oracle_lib.Oracle(game, 1)
    orc.reset(np.zeros((1, 2), np.uint32))
    C = game.bucket.per_player_capacity
    carry = oracle_lib.empty_carry(1, C)
    commands = orc.bot_act(0, oracle_lib.WORKER_RUSH, -1, carry)
    assert commands[0, :, 0, 0].tolist() == [0, -1, 10, -1, -1, 0]
    assert (carry["kind"] == -1).all() and carry["next_order"][0] == 0


def test_config4_duel_runs_to_a_decision(oracle_lib):
    """WorkerRush (player 0) against LightRush (player 1) on basesWorkers16x16:
    state invariants hold every step and the game ends with a winner; identical
    lanes stay identical.  The ending step and winner are a regression pin of
    this oracle, not an independent reference value."""
    from nanorts_b200.content import map_name_to_scenario
    from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion

    game = map_name_to_scenario("basesWorkers16x16", utt=UnitTypeTableVersion.ORIGINAL,
                                conflict_strategy=ConflictStrategy.CANCEL_BOTH, max_cycles=5000)
    orc = oracle_lib.Oracle(game, 2)
    orc.reset(np.array([[0, 0], [7, 9]], np.uint32))
    C = game.bucket.per_player_capacity
    carries = (oracle_lib.empty_carry(2, C), oracle_lib.empty_carry(2, C))
    for step in range(5000):
        out = orc.duel_step((oracle_lib.WORKER_RUSH, oracle_lib.BARRACKS_RUSH), (-1, oracle_lib.TYPE_LIGHT), carries)
        if step % 25 == 0:
            assert state_invariants(orc.state, game.bucket) == []
        for name, leaf in orc.state.items():
            assert np.array_equal(leaf[0], leaf[1]), name
        if out["done"][0]:
            break
    assert out["terminated"][0] and out["winner"][0] == 0 and step == 469
    # The carries restart empty with the new episode.
    assert (carries[0]["kind"] == -1).all() and (carries[1]["next_order"] == 0).all()
    assert orc.episode_index.tolist() == [1, 1]
