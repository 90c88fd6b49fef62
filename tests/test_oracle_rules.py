"""Known-answer tests of the CPU oracle against the rules as the reference
states them (README.md "Actions", "Gotchas"; core/reservations.py,
core/completion.py, core/kinds/*.py), on hand-built scenarios.  These pin
the oracle that the GPU parity tests then hold the kernel to."""

from __future__ import annotations

import numpy as np
import pytest

from nanorts_b200.model import ConflictStrategy
from tests.helpers import DOWN, LEFT, RIGHT, CommandSheet, idle, state_invariants, tiny_game


@pytest.fixture(scope="module")
def Oracle(oracle_lib):
    return oracle_lib.Oracle


def two_workers(strategy, **kw):
    # p0 workers at (0,0) and (2,0), both able to move into (1,0); p1 worker at (3,3).
    return tiny_game([("Worker", 0, 0, 0, 1, 0), ("Worker", 0, 2, 0, 1, 0), ("Worker", 1, 3, 3, 1, 0)],
                     strategy=strategy, **kw)


def start(Oracle, game, lanes=1, keys=None):
    orc = Oracle(game, lanes)
    orc.reset(np.zeros((lanes, 2), np.uint32) if keys is None else keys)
    return orc


def run_idle(orc, game, steps, key=(0, 0)):
    for _ in range(steps):
        orc.core_step(idle(game), np.array([key], np.uint32))


def test_cancel_both_same_cycle_claims():
    """Two MOVEs into one cell in the same cycle: both become NONE for the
    shorter duration (CANCEL_BOTH, reservations.py:169-228)."""
    from oracle.oracle import Oracle as O

    game = two_workers(ConflictStrategy.CANCEL_BOTH)
    orc = start(O, game)
    cmd = CommandSheet(game).set(0, 0, "move", direction=RIGHT).set(0, 1, "move", direction=LEFT).array
    orc.core_step(cmd, np.zeros((1, 2), np.uint32))
    s = orc.state
    assert list(s["pending_kind"][0, :2]) == [0, 0]  # both NONE
    assert list(s["pending_none_duration"][0, :2]) == [10, 10]
    assert list(s["pending_completes_at"][0, :2]) == [10, 10]
    assert list(s["pending_order"][0, :2]) == [0, 1]
    run_idle(orc, game, 9)
    assert list(s["pending_kind"][0, :2]) == [-1, -1]
    assert list(s["cell"][0, :2]) == [0, 2]  # nobody moved
    assert s["entity_at"][0].reshape(-1)[1] == -1


def test_cross_cycle_claim_is_dropped():
    """A request for a cell an earlier action already claims becomes NONE with
    duration -1 and completes at once (reservations.py:183-187)."""
    from oracle.oracle import Oracle as O

    game = two_workers(ConflictStrategy.CANCEL_BOTH)
    orc = start(O, game)
    orc.core_step(CommandSheet(game).set(0, 0, "move", direction=RIGHT).set(0, 1, "none").array, np.zeros((1, 2), np.uint32))
    s = orc.state
    assert s["pending_kind"][0, 0] == 1 and s["pending_completes_at"][0, 0] == 10
    assert s["pending_kind"][0, 1] == -1  # the 1-cycle NONE already completed
    orc.core_step(CommandSheet(game).set(0, 1, "move", direction=LEFT).array, np.zeros((1, 2), np.uint32))
    assert s["pending_kind"][0, 1] == -1  # dropped: NONE for -1 cycles, cleared the same step
    assert s["pending_kind"][0, 0] == 1  # the holder keeps its MOVE
    run_idle(orc, game, 8)
    assert s["cell"][0, 0] == 1 and s["entity_at"][0].reshape(-1)[1] == 0


def test_cancel_alternating_turns():
    """CANCEL_ALTERNATING cancels the request when (count + before) is even and
    advances the count by the same-cycle conflicts (reservations.py:207-259)."""
    from oracle.oracle import Oracle as O

    game = two_workers(ConflictStrategy.CANCEL_ALTERNATING)
    orc = start(O, game)
    cmd = CommandSheet(game).set(0, 0, "move", direction=RIGHT).set(0, 1, "move", direction=LEFT).array
    orc.core_step(cmd, np.zeros((1, 2), np.uint32))
    s = orc.state
    assert s["alternating_conflict_count"][0] == 1
    assert s["pending_kind"][0, 0] == 1  # the earlier request (holder) keeps its MOVE
    assert s["pending_kind"][0, 1] == 0 and s["pending_none_duration"][0, 1] == 10
    run_idle(orc, game, 9)
    assert list(s["cell"][0, :2]) == [1, 2]


def test_cancel_random_follows_the_conflict_draw(oracle_lib):
    """CANCEL_RANDOM cancels the request when its draw is 0, with the draw keyed
    by fold_in(fold_in(fold_in(episode key, time), birth), 0) and the ordinal."""
    from oracle.oracle import Oracle as O

    game = two_workers(ConflictStrategy.CANCEL_RANDOM)
    lib = oracle_lib.lib()
    seen = set()
    for seed in range(16):
        key = np.array([[seed * 7919 + 1, seed]], np.uint32)
        orc = start(O, game, keys=key)
        cmd = CommandSheet(game).set(0, 0, "move", direction=RIGHT).set(0, 1, "move", direction=LEFT).array
        orc.core_step(cmd, key)
        draw = lib.oracle_conflict_draw(int(key[0, 0]), int(key[0, 1]), 0, 1, 0)  # time 0, birth of the request 1
        s = orc.state
        if draw == 0:  # request cancelled, holder keeps MOVE
            assert s["pending_kind"][0, 0] == 1 and s["pending_kind"][0, 1] == 0
        else:  # holder cancelled, request admitted
            assert s["pending_kind"][0, 0] == 0 and s["pending_kind"][0, 1] == 1
        seen.add(draw)
    assert seen == {0, 1}


def test_produce_spawns_in_lowest_free_slot():
    """PRODUCE pays on completion and spawns in the lowest free slot of the
    player's block with the next birth (produce.py:49-89, units.py:12-19)."""
    from oracle.oracle import Oracle as O

    game = tiny_game([("Base", 0, 1, 1, 10, 0), ("Worker", 1, 3, 3, 1, 0)], resources=(5, 5))
    orc = start(O, game)
    cmd = CommandSheet(game).set(0, 0, "produce", direction=RIGHT, produced=3).array
    orc.core_step(cmd, np.zeros((1, 2), np.uint32))
    s = orc.state
    assert s["pending_kind"][0, 0] == 4 and s["pending_completes_at"][0, 0] == 50
    run_idle(orc, game, 48)
    assert s["birth"][0, 1] == -1 and s["player_resources"][0, 0] == 5
    run_idle(orc, game, 1)
    assert s["birth"][0, 1] == 2  # next_birth after two placed units
    assert s["unit_type"][0, 1] == 3 and s["owner"][0, 1] == 0 and s["cell"][0, 1] == 1 * 4 + 2
    assert s["hit_points"][0, 1] == 1 and s["player_resources"][0, 0] == 4 and s["next_birth"][0] == 3


def test_harvest_then_return_credits_the_player():
    from oracle.oracle import Oracle as O

    game = tiny_game([("Resource", -1, 0, 0, 1, 3), ("Worker", 0, 1, 0, 1, 0), ("Base", 0, 2, 0, 10, 0),
                      ("Worker", 1, 3, 3, 1, 0)], resources=(0, 0))
    N = game.bucket.neutral_capacity
    orc = start(O, game)
    orc.core_step(CommandSheet(game).set(0, 0, "harvest", direction=LEFT).array, np.zeros((1, 2), np.uint32))
    run_idle(orc, game, 19)
    s = orc.state
    assert s["carried_resources"][0, N] == 1 and s["carried_resources"][0, 0] == 2
    orc.core_step(CommandSheet(game).set(0, 0, "return", direction=RIGHT).array, np.zeros((1, 2), np.uint32))
    run_idle(orc, game, 9)
    assert s["carried_resources"][0, N] == 0 and s["player_resources"][0, 0] == 1


def test_attack_kills_and_decides_the_game():
    """An attack that drops hit points to 0 removes the unit; a player without
    units loses: +1 / -1 (attack.py:78-102, outcome.py:11-37)."""
    from oracle.oracle import Oracle as O

    game = tiny_game([("Worker", 0, 0, 0, 1, 0), ("Worker", 1, 1, 0, 1, 0)])
    orc = start(O, game)
    out = orc.core_step(CommandSheet(game).set(0, 0, "attack", target=1).array, np.zeros((1, 2), np.uint32))
    assert not out["terminated"][0]
    for _ in range(4):
        out = orc.core_step(idle(game), np.zeros((1, 2), np.uint32))
    s = orc.state
    assert out["terminated"][0] and not out["truncated"][0]
    assert list(out["reward"][0]) == [1.0, -1.0]
    assert s["winner"][0] == 0 and s["birth"][0, game.bucket.per_player_capacity] == -1
    assert s["entity_at"][0].reshape(-1)[1] == -1


def test_time_limit_is_a_draw():
    from oracle.oracle import Oracle as O

    game = two_workers(ConflictStrategy.CANCEL_BOTH, max_cycles=3)
    orc = start(O, game)
    outs = [orc.core_step(idle(game), np.zeros((1, 2), np.uint32)) for _ in range(3)]
    assert not outs[1]["truncated"][0]
    assert outs[2]["truncated"][0] and not outs[2]["terminated"][0]
    assert list(outs[2]["reward"][0]) == [-1.0, -1.0]


def test_env_step_decodes_rows_and_auto_resets(oracle_lib):
    """The JaxMARL step: attack offsets decode relative to the unit; unknown
    kinds become NONE for 0 cycles; finished games restart at episode + 1."""
    game = two_workers(ConflictStrategy.CANCEL_BOTH, max_cycles=2)
    orc = oracle_lib.Oracle(game, 1)
    orc.reset(np.array([[3, 4]], np.uint32))
    C = game.bucket.per_player_capacity
    actions = np.zeros((1, 2, C, 7), np.int32)
    actions[0, 0, 0] = [9, 0, 0, 0, 0, 0, 0]  # unknown kind
    out = orc.step(actions)
    assert orc.state["pending_kind"][0, 0] == -1  # NONE for 0 cycles, completed the same step
    assert not out["done"][0]
    out = orc.step(np.zeros((1, 2, C, 7), np.int32))
    assert out["done"][0] and out["truncated"][0]
    assert orc.episode_index[0] == 1 and orc.state["time"][0] == 0
    assert list(orc.environment_root[0]) == [3, 4]


def test_random_play_keeps_the_state_invariants(oracle_lib):
    from tests.parity import CONFIGS, sample

    for name in ("c1_8x8_both", "c2_16x16_random", "c3_16x16_alternating_partial"):
        cfg = CONFIGS[name]
        game = cfg.game(120)
        orc = oracle_lib.Oracle(game, 16, partial_observability=cfg.partial)
        rng = np.random.default_rng(0)
        orc.reset(rng.integers(0, 2**32, size=(16, 2), dtype=np.uint64).astype(np.uint32))
        for _ in range(150):
            orc.step(sample(orc.legal_masks(), rng, move_bias=0.3))
        assert state_invariants(orc.state, game.bucket) == []


def test_masks_of_the_reset_state():
    """bases8x8 opening: the base may produce a worker into free neighbours, the
    worker may move, harvest is not legal yet, busy and empty slots hold only NONE."""
    from oracle.oracle import Oracle as O

    from nanorts_b200 import map_name_to_scenario

    game = map_name_to_scenario("basesWorkers8x8", utt="VERSION_ORIGINAL")
    orc = O(game, 1)
    orc.reset(np.zeros((1, 2), np.uint32))
    masks = orc.legal_masks()[0]
    base, worker = masks[0, 0], masks[0, 1]  # p0: Base (2,1) in slot 0, Worker (1,1) in slot 1
    assert list(base[:6]) == [1, 0, 0, 0, 1, 0]  # NONE, PRODUCE
    assert list(base[22:29]) == [0, 0, 0, 1, 0, 0, 0]  # Worker only
    assert list(base[18:22]) == [1, 1, 1, 0]  # produce: up, right, down free; left holds the worker
    assert list(worker[:6]) == [1, 1, 0, 0, 1, 0]  # NONE, MOVE, PRODUCE (a Barracks costs 5 <= 5; a Base 10)
    assert list(worker[22:29]) == [0, 0, 1, 0, 0, 0, 0]
    assert list(masks[0, 2]) == [1] + [0] * 77  # empty slot


def test_down_is_plus_width():
    from oracle.oracle import Oracle as O

    game = tiny_game([("Worker", 0, 1, 1, 1, 0), ("Worker", 1, 3, 3, 1, 0)])
    orc = start(O, game)
    orc.core_step(CommandSheet(game).set(0, 0, "move", direction=DOWN).array, np.zeros((1, 2), np.uint32))
    run_idle(orc, game, 9)
    assert orc.state["cell"][0, 0] == 2 * 4 + 1


def test_reward_components_count_admitted_requests(oracle_lib):
    """adapters/rewards.py:47-72 over admission.py:273-296 counts: one harvest,
    one worker produced and one attack on the opponent for player 0; nothing
    for player 1; win_loss 0 while the game runs."""
    import numpy as np

    from tests.helpers import tiny_game

    game = tiny_game([("Resource", -1, 0, 1, 1, 10), ("Worker", 0, 1, 1, 1, 0), ("Base", 0, 3, 3, 10, 0),
                      ("Light", 0, 4, 0, 4, 0), ("Worker", 1, 5, 0, 1, 0), ("Base", 1, 5, 5, 10, 0)],
                     width=6, height=6, resources=(10, 10))
    orc = oracle_lib.Oracle(game, 1, reward_components=True)
    orc.reset(np.zeros((1, 2), np.uint32))
    C = game.bucket.per_player_capacity
    N = game.bucket.neutral_capacity
    actions = np.zeros((1, 2, C, 7), np.int32)
    actions[..., 0] = 0
    types = orc.state["unit_type"][0]
    owner = orc.state["owner"][0]
    for s in range(N, N + C):
        if owner[s] != 0:
            continue
        local = s - N
        if types[s] == 3:  # worker: harvest the pile to its left
            actions[0, 0, local] = [2, 0, 3, 0, 0, 0, 0]
        elif types[s] == 1:  # base: produce a worker downwards
            actions[0, 0, local] = [4, 0, 0, 0, 2, 3, 0]
        elif types[s] == 4:  # light: attack the enemy worker one cell right
            actions[0, 0, local] = [5, 0, 0, 0, 0, 0, 3 * 7 + 4]
    out = orc.step(actions)
    comp = out["reward_components"][0]
    assert comp[0].tolist() == [0.0, 1.0, 1.0, 0.0, 1.0, 0.0]
    assert comp[1].tolist() == [0.0] * 6
