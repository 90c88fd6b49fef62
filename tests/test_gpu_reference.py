"""Parity pinned to the reference itself: NanoRTS's own CUDA kernels (needs a B200).

``oracle/_ref/libref_kernels.so`` holds the reference's ``nanorts_step``,
``nanorts_legality_words``, ``nanorts_visible_cells`` and
``nanorts_reset_packed_where_done`` handlers, compiled unchanged from the
reference sources (``oracle/ref_kernels.cu``).  Along a recorded trajectory of
uniform legal play (move-biased, so claims collide) every step checks:

* the reference's core step (its kernel, fed the Commands ``decode_actions``
  gives and the episode root key) against the oracle's ``core_step``: all 23
  State leaves of every game;
* the reference's legality words, assembled as ``legal_actions`` does, against
  the oracle's rows and the product's ``get_avail_actions``;
* the reference's visible cells (partial observability) against the oracle's;
* the reference's auto-reset kernel against the oracle's reset rows;
* the product's ``nrts_step`` against the reference's step on every game the
  step did not end (an ended game is reset in place by ``nrts_step``).
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
