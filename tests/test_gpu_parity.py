"""Kernel vs oracle, bit for bit, at every step (needs a B200).

Every State leaf, both players' legality rows, feature maps and scalars,
rewards, dones, winners and telemetry of the sm_100a path are compared with
the CPU oracle's on the same seeded action stream, including episodes that
end and auto-reset inside the run (short horizons force truncation).
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


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.cpu().numpy()


def compare_state(env_state, orc, where: str) -> None:
    core = env_state.core_state
    for name in LEAVES:
        got = _np(getattr(core, name))
        want = orc.state[name]
        if got.dtype == np.bool_:
            want = want.astype(bool)
        if not np.array_equal(got, want.reshape(got.shape)):
            bad = np.argwhere(got != want.reshape(got.shape))[:5]
            raise AssertionError(f"{where}: leaf {name} differs at {bad.tolist()}")
    assert np.array_equal(_np(env_state.episode_index).astype(np.uint32), orc.episode_index), f"{where}: episode_index"
    assert np.array_equal(_np(env_state.environment_root).astype(np.uint32), orc.environment_root), f"{where}: root"


def compare_obs(obs, want, where: str, prefix: str = "") -> None:
    for p, agent in enumerate(("player_0", "player_1")):
        fm = _np(obs[agent].feature_maps)
        sc = _np(obs[agent].scalars)
        wf, ws = want[prefix + "feature_maps"][:, p], want[prefix + "scalars"][:, p]
        if not np.array_equal(fm, wf):
            bad = np.argwhere(fm != wf)[:5]
            raise AssertionError(f"{where}: {prefix}feature_maps of {agent} differ at {bad.tolist()}")
        assert np.array_equal(sc, ws), f"{where}: {prefix}scalars of {agent}"


def compare_masks(env, env_state, orc, where: str) -> np.ndarray:
    masks = env.get_avail_actions(env_state)
    want = orc.legal_masks()
    for p, agent in enumerate(("player_0", "player_1")):
        got = _np(masks[agent]).astype(np.uint8)
        if not np.array_equal(got, want[:, p]):
            bad = np.argwhere(got != want[:, p])[:5]
            raise AssertionError(f"{where}: masks of {agent} differ at {bad.tolist()}")
    return want


def run_parity(config_name: str, lanes: int, steps: int, seed: int, *, max_cycles: int | None = None,
               move_bias: float = 0.0, final_observation: bool = True, reward_components: bool = False,
               game=None) -> dict:
    from nanorts_b200.env import make
    from oracle.oracle import Oracle

    cfg = CONFIGS[config_name]
    game = cfg.game(max_cycles) if game is None else game
    env = make("NanoRTS", scenario=game, partial_observability=cfg.partial, final_observation=final_observation,
               reward_components=reward_components)
    orc = Oracle(game, lanes, partial_observability=cfg.partial, final_observation=final_observation,
                 reward_components=reward_components)
    rng = np.random.default_rng(seed)
    keys = random_keys(rng, lanes)
    obs, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    want_obs = orc.reset(keys)
    compare_state(state, orc, "reset")
    compare_obs(obs, want_obs, "reset")
    episodes, overflowed = 0, 0
    nonzero = {"any": 0, "attack": 0, "win_loss": 0}
    for t in range(steps):
        masks = compare_masks(env, state, orc, f"step {t} masks")
        actions = sample(masks, rng, move_bias)
        want = orc.step(actions)
        acts = {f"player_{p}": torch.from_numpy(np.ascontiguousarray(actions[:, p])).cuda() for p in range(2)}
        obs, state, rewards, dones, infos = env.step(None, state, acts)
        where = f"{config_name} step {t}"
        compare_state(state, orc, where)
        compare_obs(obs, want, where)
        if final_observation:
            compare_obs(infos["final_observation"], want, where, prefix="final_")
        for p in range(2):
            assert np.array_equal(_np(rewards[f"player_{p}"]), want["reward"][:, p]), f"{where}: reward {p}"
        assert np.array_equal(_np(dones["__all__"]), want["done"]), f"{where}: done"
        assert np.array_equal(_np(infos["terminated"]), want["terminated"]), f"{where}: terminated"
        assert np.array_equal(_np(infos["truncated"]), want["truncated"]), f"{where}: truncated"
        assert np.array_equal(_np(infos["winner"]), want["winner"]), f"{where}: winner"
        assert np.array_equal(_np(infos["telemetry"].spawn_overflow), want["spawn_overflow"]), f"{where}: overflow"
        if reward_components:
            for p, agent in enumerate(("player_0", "player_1")):
                got = _np(infos["reward_components"][agent])
                if not np.array_equal(got, want["reward_components"][:, p]):
                    bad = np.argwhere(got != want["reward_components"][:, p])[:5]
                    raise AssertionError(f"{where}: reward_components of {agent} differ at {bad.tolist()}")
            nonzero["any"] += int(np.count_nonzero(want["reward_components"][..., 1:]))
            nonzero["attack"] += int(np.count_nonzero(want["reward_components"][..., 4]))
            nonzero["win_loss"] += int(np.count_nonzero(want["reward_components"][..., 0]))
        episodes += int(want["done"].sum())
        overflowed += int((want["spawn_overflow"] > 0).any(axis=1).sum())
    return {"episodes": episodes, "time": orc.state["time"].copy(), "alt": orc.state["alternating_conflict_count"].copy(),
            "components": nonzero, "overflowed": overflowed}


@pytest.mark.parametrize("config_name", ["c1_8x8_both", "c2_16x16_random", "c3_16x16_alternating_partial"])
def test_parity_small_boards(config_name):
    stats = run_parity(config_name, lanes=96, steps=400, seed=1, max_cycles=150)
    assert stats["episodes"] > 0  # auto-reset exercised


@pytest.mark.parametrize("config_name", ["c2_16x16_random", "c3_16x16_alternating_partial", "c1_8x8_both"])
def test_parity_contested_moves(config_name):
    """Move-biased play: many same-cycle and cross-cycle claim conflicts."""
    stats = run_parity(config_name, lanes=64, steps=300, seed=7, move_bias=0.7, max_cycles=120)
    if config_name.startswith("c3"):
        assert stats["alt"].max() > 0  # CANCEL_ALTERNATING counted conflicts


@pytest.mark.parametrize("config_name,lanes", [("c2_16x16_random", 4096), ("c1_8x8_both", 4400),
                                               ("c3_16x16_alternating_partial", 3600), ("c2_16x16_random", 2000)])
def test_parity_full_batches(config_name, lanes):
    """Batches that fill every SM: from about 3400 games on 16 x 16 the launch
    holds one CTA of up to 28 games per SM (a persistent grid); 2000 games take
    CTAs of up to 8 games.  (Small batches, as in the other tests, run one game
    per CTA of 2 or 4 warps.)"""
    stats = run_parity(config_name, lanes=lanes, steps=60, seed=17, max_cycles=40, move_bias=0.3)
    assert stats["episodes"] > 0


@pytest.mark.parametrize("config_name", ["c5_64x64_random", "c5_64x64_alternating_partial"])
def test_parity_garden_of_war(config_name):
    """64 x 64 boards: one game per CTA, its outputs written by every warp."""
    stats = run_parity(config_name, lanes=12, steps=200, seed=3, max_cycles=90, move_bias=0.3,
                       reward_components=True)
    assert stats["episodes"] > 0


def test_parity_long_horizon():
    """Games that run long enough for units to fight and die (default horizon)."""
    run_parity("c2_16x16_random", lanes=48, steps=1200, seed=11, final_observation=False)


def test_parity_long_horizon_config3():
    """Config 3 (fine-tuned table, CANCEL_ALTERNATING, partial observability)
    at its default horizon: 2000 steps of 64 games."""
    stats = run_parity("c3_16x16_alternating_partial", lanes=64, steps=2000, seed=23, final_observation=False)
    print(f"config 3: {stats['episodes']} games ended in 2000 steps")
    assert stats["alt"].max() > 0


def test_parity_long_horizon_config5():
    """Config 5 (GardenOfWar64x64, CANCEL_RANDOM) for 3000 steps of 8 games."""
    stats = run_parity("c5_64x64_random", lanes=8, steps=3000, seed=29, final_observation=False, move_bias=0.1)
    print(f"config 5: {stats['episodes']} games ended in 3000 steps")


def test_parity_spawn_overflow():
    """A player block of 3 slots on basesWorkers8x8: production runs out of
    slots, the kernel counts spawn_overflow (core/kinds/produce.py:55-75) as
    the oracle does, and the telemetry turns nonzero."""
    from nanorts_b200.content import assemble_game, shipped_document
    from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion

    game = assemble_game(shipped_document("basesWorkers8x8"), utt=UnitTypeTableVersion.ORIGINAL,
                         conflict_strategy=ConflictStrategy.CANCEL_BOTH, max_cycles=400, per_player_capacity=3)
    assert game.bucket.per_player_capacity == 3
    stats = run_parity("c1_8x8_both", lanes=48, steps=500, seed=37, move_bias=0.6, game=game)
    print(f"spawn overflow: {stats['overflowed']} game-steps with a nonzero counter")
    assert stats["overflowed"] > 0


def test_parity_garden_of_war_production_shape():
    """Config 5's launch as the benchmark runs it: 1,500 GardenOfWar64x64
    games on the persistent grid of step_kernel_wide<64> (3 CTAs per SM, 444
    on a B200, so every CTA steps about 3 games and prefetches the next one
    into L2), the fused draw on, the game order reversed every other launch,
    and a horizon of 20 so every game resets inside the run.  (On 8x8 and
    16x16 boards a team launch is chosen only when the whole batch is
    resident at once, so games never outnumber CTAs there.)"""
    from nanorts_b200.env import make
    from oracle.oracle import Oracle

    cfg = CONFIGS["c5_64x64_random"]
    game = cfg.game(20)
    lanes = 1500
    env = make("NanoRTS", scenario=game, final_observation=False)
    orc = Oracle(game, lanes)
    rng = np.random.default_rng(41)
    keys = random_keys(rng, lanes)
    obs, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    compare_obs(obs, orc.reset(keys), "reset")
    actions = env.sample_actions(state, seed=3, counter=0)
    episodes = 0
    for t in range(30):
        host = np.stack([_np(actions[a]) for a in ("player_0", "player_1")], 1)
        want = orc.step(host)
        obs, state, rewards, dones, infos = env.step(None, state, {a: actions[a].clone() for a in actions},
                                                     sample=(3, t + 1))
        where = f"production shape step {t}"
        compare_state(state, orc, where)
        compare_obs(obs, want, where)
        assert np.array_equal(_np(dones["__all__"]), want["done"]), f"{where}: done"
        assert np.array_equal(_np(rewards["player_0"]), want["reward"][:, 0]), f"{where}: reward"
        if t % 10 == 9:
            compare_masks(env, state, orc, where)
        episodes += int(want["done"].sum())
        actions = {a: infos["sampled_actions"][a].clone() for a in ("player_0", "player_1")}
    assert episodes >= lanes


@pytest.mark.parametrize("config_name", ["c2_16x16_random", "c1_8x8_both"])
def test_parity_reward_components(config_name):
    """reward_components=True (adapters/rewards.py:47-72): every component of
    both players at every step, over games long enough to fight and end."""
    stats = run_parity(config_name, lanes=64, steps=700, seed=13, move_bias=0.3, final_observation=False,
                       reward_components=True)
    assert stats["components"]["any"] > 0 and stats["components"]["attack"] > 0


@pytest.mark.parametrize("config_name", ["c2_16x16_random", "c5_64x64_random", "c1_8x8_both"])
def test_fused_sampler_matches_standalone_and_oracle(config_name):
    """Actions drawn inside nrts_step equal nrts_sample_actions' on the same
    rows, and stepping on them keeps the kernel equal to the oracle."""
    from nanorts_b200.env import make
    from oracle.oracle import Oracle

    cfg = CONFIGS[config_name]
    game = cfg.game(200)
    lanes = {"c2": 128, "c5": 8, "c1": 13}[config_name[:2]]  # c1: 611 rows, a partial 32-row chunk
    env = make("NanoRTS", scenario=game, final_observation=False)
    orc = Oracle(game, lanes)
    rng = np.random.default_rng(5)
    keys = random_keys(rng, lanes)
    _, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    orc.reset(keys)
    actions = env.sample_actions(state, seed=9, counter=0)
    for t in range(250):
        host = np.stack([_np(actions[a]) for a in ("player_0", "player_1")], 1)
        want = orc.step(host)
        acts = {a: actions[a].clone() for a in actions}
        obs, state, rewards, dones, infos = env.step(None, state, acts, sample=(9, t + 1))
        compare_state(state, orc, f"fused step {t}")
        assert np.array_equal(_np(dones["__all__"]), want["done"])
        fused = {a: infos["sampled_actions"][a].clone() for a in ("player_0", "player_1")}
        env.invalidate(state)  # recompute the rows with nrts_legal_masks, then draw with the standalone kernel
        standalone = env.sample_actions(state, seed=9, counter=t + 1)
        for a in fused:
            assert torch.equal(fused[a], standalone[a]), f"step {t}: fused draw differs for {a}"
        actions = fused


def test_standalone_sampler_reads_any_nonzero_byte_at_any_alignment():
    """nrts_sample_actions: a row byte is legal when nonzero, and mask arrays
    that do not start on a 16-byte boundary draw the same actions."""
    import ctypes

    from nanorts_b200.env import _ptr, make
    from nanorts_b200.runtime import check, library

    game = CONFIGS["c2_16x16_random"].game(100)
    lanes, C = 37, game.bucket.per_player_capacity
    env = make("NanoRTS", scenario=game, final_observation=False)
    rng = np.random.default_rng(3)
    keys = random_keys(rng, lanes)
    _, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    for t in range(20):
        env.step(None, state, env.sample_actions(state, seed=1, counter=t))
    want = {a: v.clone() for a, v in env.sample_actions(state, seed=4, counter=77).items()}
    masks = env._row_masks(state)
    width = masks["player_0"].shape[-1]

    def draw(m0, m1):
        out = torch.empty((2, lanes, C, 7), dtype=torch.int32, device="cuda")
        check(library().nrts_sample_actions(ctypes.byref(env._extents), lanes, _ptr(m0), _ptr(m1), _ptr(out[0]),
                                            _ptr(out[1]), 4, 77, env._stream()))
        return out

    scaled = [(masks[a].view(torch.uint8) * torch.randint(1, 255, masks[a].shape, device="cuda", dtype=torch.uint8)
               * (masks[a].view(torch.uint8) != 0)).contiguous() for a in ("player_0", "player_1")]
    got = draw(scaled[0], scaled[1])
    for p, a in enumerate(("player_0", "player_1")):
        assert torch.equal(got[p], want[a]), f"nonzero bytes: {a}"
    n = lanes * C * width
    for shift in (1, 5, 8):
        buf = torch.zeros((2, n + 16), dtype=torch.uint8, device="cuda")
        buf[0, shift:shift + n] = masks["player_0"].reshape(-1).view(torch.uint8)
        buf[1, shift:shift + n] = masks["player_1"].reshape(-1).view(torch.uint8)
        got = draw(buf[0, shift:], buf[1, shift:])
        for p, a in enumerate(("player_0", "player_1")):
            assert torch.equal(got[p], want[a]), f"shift {shift}: {a}"


def pack_rows(rows: np.ndarray, widths: tuple[int, ...]) -> np.ndarray:
    """adapters/factors.py:89-103 pack, on uint8 [..., 78] rows."""
    head = sum(widths[:-1])
    middle = head + min(widths[-1], 32)
    words = []
    for start, stop in ((0, head), (head, middle), (middle, head + widths[-1])):
        shifts = np.arange(stop - start, dtype=np.uint64)
        words.append((rows[..., start:stop].astype(np.uint64) << shifts).sum(-1).astype(np.uint32))
    return np.stack(words, -1)


@pytest.mark.parametrize("config_name", ["c2_16x16_random", "c5_64x64_random"])
def test_packed_masks_match_the_oracle_rows(config_name):
    """mask_form='packed': the step's packed words, nrts_packed_masks on a
    state it did not produce, and their unpacking all equal the oracle's rows."""
    from nanorts_b200.env import make, unpack_mask
    from oracle.oracle import Oracle

    cfg = CONFIGS[config_name]
    game = cfg.game(100)
    lanes = 32 if config_name.startswith("c2") else 6
    env = make("NanoRTS", scenario=game, final_observation=False, mask_form="packed")
    assert env.layout.mask_shape == (game.bucket.per_player_capacity, 3)
    orc = Oracle(game, lanes)
    rng = np.random.default_rng(21)
    keys = random_keys(rng, lanes)
    _, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    orc.reset(keys)
    widths = env.layout.action_widths
    for t in range(150):
        want_rows = orc.legal_masks()
        words = env.get_avail_actions(state)
        for p, agent in enumerate(("player_0", "player_1")):
            got = words[agent].view(torch.int32).cpu().numpy().view(np.uint32)
            assert np.array_equal(got, pack_rows(want_rows[:, p], widths)), f"step {t}: packed words of {agent}"
            assert np.array_equal(unpack_mask(words[agent], env.layout).cpu().numpy(), want_rows[:, p].astype(bool))
        if t % 25 == 0:  # the standalone entry point on the same state
            env.invalidate(state)
            again = env.get_avail_actions(state)
            for agent in again:
                assert torch.equal(again[agent], words[agent].clone()), f"step {t}: nrts_packed_masks differs"
        actions = sample(want_rows, rng, 0.3)
        orc.step(actions)
        acts = {f"player_{p}": torch.from_numpy(np.ascontiguousarray(actions[:, p])).cuda() for p in range(2)}
        env.step(None, state, acts)
        compare_state(state, orc, f"packed step {t}")
