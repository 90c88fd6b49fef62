"""Parity pinned to the reference itself: NanoRTS's own CUDA kernels (needs a B200).

``oracle/_ref/libref_kernels.so`` holds the reference's ``nanorts_step``,
``nanorts_legality_words``, ``nanorts_visible_cells``,
``nanorts_reset_packed_where_done`` and ``nanorts_abstraction_act`` handlers,
compiled unchanged from the reference sources (``oracle/ref_kernels.cu``).  Along a recorded trajectory of
uniform legal play (move-biased, so claims collide) every step checks:

* the reference's core step (its kernel, fed the Commands ``decode_actions``
  gives and the episode root key) against the oracle's ``core_step``: all 23
  State leaves of every game;
* the reference's legality words, assembled as ``legal_actions`` does, against
  the oracle's rows and the product's ``get_avail_actions``;
* the reference's visible cells (partial observability) against the oracle's;
* the reference's auto-reset kernel against the oracle's reset rows;
* the product's ``nrts_step`` against the reference's step on every game the
  step did not end (an ended game is reset in place by ``nrts_step``);
* config 4's rush bots: the reference's bot kernel against the oracle's and
  the product's Commands and carries.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.parity import CONFIGS, random_keys, sample

pytestmark = pytest.mark.gpu

LEAVES = (
    "birth", "unit_type", "owner", "cell", "hit_points", "carried_resources", "pending_kind", "pending_direction",
    "pending_none_duration", "pending_target_cell", "pending_produced_type", "pending_issued_at",
    "pending_completes_at", "pending_order", "entity_at", "time", "player_resources", "next_birth",
    "next_pending_order", "alternating_conflict_count", "game_over", "winner", "spawn_overflow",
)


def _reference():
    from oracle import ref_kernels

    if not ref_kernels.available():
        pytest.skip("the reference kernels are not built (make -C oracle ref with a NanoRTS checkout)")
    return ref_kernels


def _np(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def _upload(state: dict[str, np.ndarray]) -> dict[str, torch.Tensor]:
    return {name: torch.from_numpy(np.ascontiguousarray(state[name])).cuda() for name in LEAVES}


def _diff(got: np.ndarray, want: np.ndarray, where: str) -> None:
    want = want.reshape(got.shape).astype(got.dtype)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)[:5]
        raise AssertionError(f"{where} differs at {bad.tolist()}")


def run_reference_parity(config_name: str, lanes: int, steps: int, seed: int, *, max_cycles: int,
                         move_bias: float) -> dict:
    ref_kernels = _reference()
    from nanorts_b200.env import make
    from nanorts_b200.model import ConflictStrategy
    from oracle.oracle import Oracle

    cfg = CONFIGS[config_name]
    game = cfg.game(max_cycles)
    b = game.bucket
    ref = ref_kernels.ReferenceKernels(game)
    env = make("NanoRTS", scenario=game, partial_observability=cfg.partial, final_observation=False)
    orc = Oracle(game, lanes, partial_observability=cfg.partial)
    probe = Oracle(game, lanes)
    rng = np.random.default_rng(seed)
    keys = random_keys(rng, lanes)
    _, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    orc.reset(keys)
    packed = ref.packed_reset_rows(probe._reset)
    events = ref.event_buffers(lanes)
    draws = b.conflict_strategy == ConflictStrategy.CANCEL_RANDOM
    stats = {"episodes": 0, "conflicts": 0, "spawn_overflow": 0}
    for t in range(steps):
        where = f"{config_name} step {t}"
        leaves = _upload(orc.state)
        # Legality: the reference's words kernel, assembled as legal_actions.
        masks = orc.legal_masks()
        ref_rows = _np(ref.avail_rows(leaves)).astype(np.uint8)
        _diff(ref_rows, masks, f"{where}: reference legality vs oracle")
        got = env.get_avail_actions(state)
        for p, agent in enumerate(("player_0", "player_1")):
            _diff(_np(got[agent]).astype(np.uint8), ref_rows[:, p], f"{where}: product masks of {agent} vs reference")
        # Visibility: the reference's stamping kernel against the oracle's test.
        if cfg.partial:
            for p in range(2):
                seen = torch.empty((lanes, b.height, b.width), dtype=torch.bool, device="cuda")
                ref.visible_cells(leaves, p, seen)
                _diff(_np(seen), orc.visible_cells(p), f"{where}: visible cells of player {p}")
        # Core step: the reference kernel against the oracle's core_step.
        actions = sample(masks, rng, move_bias)
        commands = orc.decode_actions(actions)
        roots = orc.episode_roots() if draws else np.zeros((lanes, 2), np.uint32)
        for name in LEAVES:
            probe.state[name][...] = orc.state[name]
        probe.environment_root[...] = orc.environment_root
        probe.episode_index[...] = orc.episode_index
        outcome = probe.core_step(commands, roots)
        rows = [torch.from_numpy(np.ascontiguousarray(commands[:, k])).cuda() for k in range(6)]
        counters = {name: torch.empty_like(leaves[name]) for name in ref_kernels.COUNTERS}
        ref.step(leaves, counters, rows, torch.from_numpy(roots.view(np.int32)).cuda(), events)
        stepped = {**{n: leaves[n] for n in ref_kernels.ROWS}, **counters}
        for name in LEAVES:
            _diff(_np(stepped[name]), probe.state[name], f"{where}: reference step leaf {name} vs oracle")
        # The product's full step (core step, auto-reset, outputs) on the same actions.
        want = orc.step(actions)
        acts = {f"player_{p}": torch.from_numpy(np.ascontiguousarray(actions[:, p])).cuda() for p in range(2)}
        _, state, _, dones, _ = env.step(None, state, acts)
        done = want["done"]
        assert np.array_equal(_np(dones["__all__"]), done), f"{where}: done"
        assert np.array_equal(done, outcome["terminated"] | outcome["truncated"]), f"{where}: oracle outcome"
        core = state.core_state
        kept = ~done
        for name in LEAVES:
            _diff(_np(getattr(core, name))[kept], _np(stepped[name])[kept], f"{where}: product leaf {name} vs reference")
        # Auto-reset: the reference's packed reset kernel on the ended games' rows.
        ref.reset_where_done(torch.from_numpy(done).cuda(), packed, leaves)
        for name in ref_kernels.ROWS:
            _diff(_np(leaves[name]), orc.state[name], f"{where}: reference reset leaf {name} vs oracle")
        stats["episodes"] += int(done.sum())
        stats["conflicts"] = max(stats["conflicts"], int(orc.state["alternating_conflict_count"].max()))
        stats["spawn_overflow"] += int((want["spawn_overflow"] > 0).sum())
    torch.cuda.synchronize()
    return stats


@pytest.mark.parametrize("config_name,lanes,steps,max_cycles", [
    ("c1_8x8_both", 64, 300, 120),
    ("c2_16x16_random", 64, 300, 150),
    ("c3_16x16_alternating_partial", 64, 300, 150),
    ("c5_64x64_random", 6, 200, 90),
    ("c5_64x64_alternating_partial", 4, 150, 80),
])
def test_reference_kernels_pin_oracle_and_product(config_name, lanes, steps, max_cycles):
    stats = run_reference_parity(config_name, lanes, steps, seed=31, max_cycles=max_cycles, move_bias=0.5)
    assert stats["episodes"] > 0  # auto-reset exercised
    if "alternating" in config_name:
        assert stats["conflicts"] > 0


def test_reference_kernels_long_horizon():
    """Default horizon, uniform play: fights, deaths and game ends."""
    stats = run_reference_parity("c2_16x16_random", 32, 900, seed=5, max_cycles=5000, move_bias=0.0)
    assert stats is not None


@pytest.mark.parametrize("config", ["c4_16x16_both", "obstacle8x8_random", "letmeout_alternating", "itsnotsafe_both",
                                    "fourbases12_random"])
def test_reference_bot_kernel_pins_oracle_and_product(config):
    """Config 4's rush bots: the reference's ``nanorts_abstraction_act`` kernel
    (WorkerRush for player 0, LightRush for player 1) against the oracle's
    ``bot_act`` and the product's ``nrts_bot_act``: the Commands and the
    settled carry of both players at every step of bot-against-bot play, from
    fresh resets and from random-play prefixes (walls, corridors, a 15-wide
    board and four bases among the maps)."""
    ref_kernels = _reference()
    from nanorts_b200.bots import Bot
    from nanorts_b200.env import make
    from oracle.oracle import empty_carry
    from tests.test_gpu_bots import BOT_CONFIGS, PAIRS, _carry_to_gpu, _compare_carry, _oracle_batch
    from tests.test_gpu_bots import _upload as upload_env

    cfg = BOT_CONFIGS[config]
    game = cfg.game(5000 if config.startswith("c4") else 400)
    bots = PAIRS["worker_vs_light"]
    orc = _oracle_batch(game, [(8, 0), (8, 20), (16, 60)], seed=19)
    L, C = orc.lanes, game.bucket.per_player_capacity
    ref = ref_kernels.ReferenceKernels(game)
    env = make("NanoRTS", scenario=game, final_observation=False)
    _, state = env.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    gpu_bots = [Bot(f"p{p}", s, t) for p, (s, t) in enumerate(bots)]
    carries = (empty_carry(L, C), empty_carry(L, C))
    ended = 0
    for step in range(500 if config.startswith("c4") else 200):
        leaves = _upload(orc.state)
        upload_env(state, orc)
        env.invalidate(state)
        for p in range(2):
            where = f"{config} step {step} player {p}"
            want_carry = {k: v.copy() for k, v in carries[p].items()}
            want = orc.bot_act(p, bots[p][0], bots[p][1], want_carry)
            ref_carry = {k: torch.from_numpy(v.copy()).cuda() for k, v in carries[p].items()}
            got = _np(ref.bot_act(leaves, p, bots[p][0], bots[p][1], ref_carry))
            _diff(got, want, f"{where}: reference commands vs oracle")
            for name, value in want_carry.items():
                _diff(_np(ref_carry[name]), value, f"{where}: reference carry {name} vs oracle")
            product_carry = _carry_to_gpu(carries[p], "cuda")
            product = _np(gpu_bots[p].act(None, product_carry, state, env, p))
            _diff(product, got, f"{where}: product commands vs reference")
            _compare_carry(product_carry, {k: _np(v) for k, v in ref_carry.items()}, f"{where}: product carry vs reference")
        want = orc.duel_step(tuple(b[0] for b in bots), tuple(b[1] for b in bots), carries)
        ended += int(want["done"].sum())
    torch.cuda.synchronize()
    if config.startswith("c4"):
        assert ended > 0, "no game ended inside the run"


@pytest.mark.parametrize("config_name,lanes", [("c1_8x8_both", 48), ("c3_16x16_alternating_partial", 48)])
def test_reference_timing_path_steps_like_the_oracle(config_name, lanes):
    """The reference path bench.py times (the reference's kernels with torch
    in place of its XLA fusions) steps games exactly as the oracle does,
    auto-reset and masks included (configs without random conflict draws,
    whose keys that path fixes)."""
    ref_kernels = _reference()
    from oracle.oracle import Oracle

    cfg = CONFIGS[config_name]
    game = cfg.game(100)
    path = ref_kernels.ReferencePath(game, lanes, partial=cfg.partial)
    orc = Oracle(game, lanes, partial_observability=cfg.partial)
    orc.reset(np.zeros((lanes, 2), np.uint32))
    rng = np.random.default_rng(3)
    for t in range(250):
        masks = orc.legal_masks()
        actions = sample(masks, rng, 0.4)
        rows = path.step(timed=False, actions=torch.from_numpy(actions).cuda())
        _diff(_np(rows).astype(np.uint8), masks, f"{config_name} step {t}: masks")
        orc.step(actions)
        for name in LEAVES:
            _diff(_np(path.leaves[name]), orc.state[name], f"{config_name} step {t}: leaf {name}")


def test_reference_duel_path_plays_like_the_oracle():
    """The reference duel path bench.py times (the reference's bot, step and
    reset kernels with torch for the seat merge, the counter select and the
    carry reset) plays config 4 exactly as the oracle's duel step does,
    through a game's end and restart."""
    ref_kernels = _reference()
    from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion
    from oracle.oracle import Oracle, empty_carry
    from tests.parity import Config

    game = Config("c4", "basesWorkers16x16", UnitTypeTableVersion.ORIGINAL, ConflictStrategy.CANCEL_BOTH).game(5000)
    bots = ((0, -1), (1, 4))
    lanes = 4
    path = ref_kernels.ReferenceDuelPath(game, lanes, bots)
    orc = Oracle(game, lanes)
    orc.reset(np.zeros((lanes, 2), np.uint32))
    C = game.bucket.per_player_capacity
    carries = (empty_carry(lanes, C), empty_carry(lanes, C))
    ended = 0
    for t in range(700):
        want = orc.duel_step((bots[0][0], bots[1][0]), (bots[0][1], bots[1][1]), carries)
        done = path.step(timed=False)
        assert np.array_equal(_np(done), want["done"]), f"step {t}: done"
        for name in LEAVES:
            _diff(_np(path.leaves[name]), orc.state[name], f"step {t}: leaf {name}")
        for p in range(2):
            for name, value in carries[p].items():
                _diff(_np(path.carries[p][name]), value, f"step {t}: carry {p} {name}")
        ended += int(want["done"].sum())
    assert ended > 0
