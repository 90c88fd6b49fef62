"""Rush bots on the sm_100a path vs the CPU oracle, bit for bit (needs a B200).

nrts_bot_act: the Commands and the settled carry of each player's bot on
states and carries taken from oracle duels (random-play prefixes make the
states differ lane to lane).  nrts_duel_step: every State leaf, both carries
and the step outputs after each step of bot-against-bot play, including games
that end and restart with empty carries.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.parity import Config, random_keys, sample
from tests.test_gpu_parity import LEAVES, _np
from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion

pytestmark = pytest.mark.gpu

O, F = UnitTypeTableVersion.ORIGINAL, UnitTypeTableVersion.ORIGINAL_FINETUNED
BOT_CONFIGS = {
    # Config 4: basesWorkers16x16, CANCEL_BOTH, WorkerRush against LightRush.
    "c4_16x16_both": Config("c4_16x16_both", "basesWorkers16x16", O, ConflictStrategy.CANCEL_BOTH),
    # Walls in the way of the searches, random conflict draws.
    "obstacle8x8_random": Config("obstacle8x8_random", "basesWorkers8x8Obstacle", O, ConflictStrategy.CANCEL_RANDOM,
                                 capacity_profile=False),
    # 8 x 16 walled corridor, alternating conflicts, the fine-tuned table.
    "letmeout_alternating": Config("letmeout_alternating", "letMeOut", F, ConflictStrategy.CANCEL_ALTERNATING,
                                   capacity_profile=False),
    # Width 15: the kernel's generic-width path.
    "itsnotsafe_both": Config("itsnotsafe_both", "itsNotSafe", O, ConflictStrategy.CANCEL_BOTH, capacity_profile=False),
    # Several bases per player: nearest-stockpile choices.
    "fourbases12_random": Config("fourbases12_random", "FourBasesWorkers12x12", O, ConflictStrategy.CANCEL_RANDOM,
                                 capacity_profile=False),
}

PAIRS = {
    "worker_vs_light": ((0, -1), (1, 4)),
    "light_vs_worker": ((1, 4), (0, -1)),
}


def _oracle_batch(game, parts, seed):
    """An oracle over the concatenation of `parts` = [(lanes, random_prefix_steps)]."""
    from oracle.oracle import LEAVES as OLEAVES, Oracle

    rng = np.random.default_rng(seed)
    pieces = []
    for lanes, prefix in parts:
        o = Oracle(game, lanes)
        o.reset(random_keys(rng, lanes))
        for _ in range(prefix):
            o.step(sample(o.legal_masks(), rng, move_bias=0.3))
        pieces.append(o)
    total = sum(p.lanes for p in pieces)
    orc = Oracle(game, total)
    for name in OLEAVES:
        orc.state[name][:] = np.concatenate([p.state[name] for p in pieces])
    orc.environment_root[:] = np.concatenate([p.environment_root for p in pieces])
    orc.episode_index[:] = np.concatenate([p.episode_index for p in pieces])
    return orc


def _upload(env_state, orc) -> None:
    core = env_state.core_state
    for name in LEAVES:
        t = getattr(core, name)
        t.copy_(torch.from_numpy(np.ascontiguousarray(orc.state[name].reshape(t.shape))))
    env_state.environment_root.copy_(torch.from_numpy(orc.environment_root.view(np.int32)).view(torch.uint32))
    env_state.episode_index.copy_(torch.from_numpy(orc.episode_index.view(np.int32)).view(torch.uint32))


def _carry_to_gpu(carry: dict, device) -> "AbstractActions":  # noqa: F821
    from nanorts_b200.bots import CARRY_FIELDS, AbstractActions

    fields = {name: torch.from_numpy(carry[name].copy()).to(device) for name in CARRY_FIELDS}
    return AbstractActions(**fields, trained=torch.from_numpy(carry["trained"].copy()).to(device),
                           next_order=torch.from_numpy(carry["next_order"].copy()).to(device))


def _compare_carry(got, want: dict, where: str) -> None:
    from nanorts_b200.bots import CARRY_FIELDS

    for name in (*CARRY_FIELDS, "trained", "next_order"):
        g = _np(getattr(got, name))
        if not np.array_equal(g, want[name]):
            bad = np.argwhere(g != want[name])[:5]
            raise AssertionError(f"{where}: carry {name} differs at {bad.tolist()} "
                                 f"(got {g[tuple(bad[0])]}, want {want[name][tuple(bad[0])]})")


def _compare_state(env_state, orc, where: str) -> None:
    core = env_state.core_state
    for name in LEAVES:
        got = _np(getattr(core, name))
        want = orc.state[name].reshape(got.shape)
        if got.dtype == np.bool_:
            want = want.astype(bool)
        if not np.array_equal(got, want):
            bad = np.argwhere(got != want)[:5]
            raise AssertionError(f"{where}: leaf {name} differs at {bad.tolist()}")
    assert np.array_equal(_np(env_state.episode_index).astype(np.uint32), orc.episode_index), f"{where}: episode_index"


@pytest.mark.parametrize("config", sorted(BOT_CONFIGS))
@pytest.mark.parametrize("pair", sorted(PAIRS))
def test_bot_act_matches_oracle(config, pair):
    from nanorts_b200.bots import Bot
    from nanorts_b200.env import make
    from oracle.oracle import empty_carry

    cfg = BOT_CONFIGS[config]
    game = cfg.game(600)
    bots = PAIRS[pair]
    orc = _oracle_batch(game, [(4, 0), (12, 20), (16, 60)], seed=11)
    L, C = orc.lanes, game.bucket.per_player_capacity
    env = make("NanoRTS", scenario=game, final_observation=False)
    _, state = env.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    carries = (empty_carry(L, C), empty_carry(L, C))
    gpu_bots = [Bot(f"p{p}", s, t) for p, (s, t) in enumerate(bots)]
    for step in range(40):
        _upload(state, orc)
        env.invalidate(state)
        for p in range(2):
            want_carry = {k: v.copy() for k, v in carries[p].items()}
            want = orc.bot_act(p, bots[p][0], bots[p][1], want_carry)
            got_carry = _carry_to_gpu(carries[p], "cuda")
            got = _np(gpu_bots[p].act(None, got_carry, state, env, p))
            torch.cuda.synchronize()
            if not np.array_equal(got, want):
                bad = np.argwhere(got != want)[:5]
                raise AssertionError(f"{config}/{pair} step {step} player {p}: commands differ at {bad.tolist()} "
                                     f"(got {got[tuple(bad[0])]}, want {want[tuple(bad[0])]})")
            _compare_carry(got_carry, want_carry, f"{config}/{pair} step {step} player {p}")
        orc.duel_step(tuple(b[0] for b in bots), tuple(b[1] for b in bots), carries)


@pytest.mark.parametrize("config", sorted(BOT_CONFIGS))
def test_duel_matches_oracle(config):
    from nanorts_b200.bots import Bot, Duel
    from nanorts_b200.env import make
    from oracle.oracle import empty_carry

    cfg = BOT_CONFIGS[config]
    full = config == "c4_16x16_both"
    game = cfg.game(5000 if full else 300)
    bots = PAIRS["worker_vs_light"]
    orc = _oracle_batch(game, [(8, 0), (8, 15), (16, 45)], seed=5)
    L, C = orc.lanes, game.bucket.per_player_capacity
    env = make("NanoRTS", scenario=game, final_observation=False)
    duel = Duel(env, (Bot("p0", *bots[0]), Bot("p1", *bots[1])))
    ds = duel.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    _upload(ds.environment_state, orc)
    carries = (empty_carry(L, C), empty_carry(L, C))
    ended = 0
    for step in range(700 if full else 360):
        want = orc.duel_step(tuple(b[0] for b in bots), tuple(b[1] for b in bots), carries)
        _, rewards, dones, infos = duel.step(ds)
        torch.cuda.synchronize()
        where = f"{config} step {step}"
        _compare_state(ds.environment_state, orc, where)
        for p in range(2):
            _compare_carry(ds.carries[p], carries[p], f"{where} player {p}")
        assert np.array_equal(_np(dones["__all__"]), want["done"]), f"{where}: done"
        assert np.array_equal(_np(infos["winner"]), want["winner"]), f"{where}: winner"
        assert np.array_equal(_np(infos["terminated"]), want["terminated"]), f"{where}: terminated"
        assert np.array_equal(_np(infos["truncated"]), want["truncated"]), f"{where}: truncated"
        assert np.array_equal(_np(infos["telemetry"].spawn_overflow), want["spawn_overflow"]), f"{where}: overflow"
        for p, agent in enumerate(("player_0", "player_1")):
            assert np.array_equal(_np(rewards[agent]), want["reward"][:, p]), f"{where}: reward {agent}"
        ended += int(want["done"].sum())
    assert ended > 0, "no game ended inside the run"


def test_duel_at_the_persistent_launch_shape_matches_oracle():
    """Full batches run one CTA per SM holding up to 20 games, each warp
    looping over every (SMs x warps)-th game: 6144 games on 148 SMs give
    most warps two or three games per launch.  Short episodes (max_cycles
    150) make games end and restart with empty carries inside the loop."""
    from nanorts_b200.bots import Bot, Duel
    from nanorts_b200.env import make
    from oracle.oracle import empty_carry

    game = BOT_CONFIGS["c4_16x16_both"].game(150)
    bots = PAIRS["light_vs_worker"]
    orc = _oracle_batch(game, [(2048, 0), (2048, 20), (2048, 60)], seed=11)
    L, C = orc.lanes, game.bucket.per_player_capacity
    assert L > 148 * 20
    env = make("NanoRTS", scenario=game, final_observation=False)
    duel = Duel(env, (Bot("p0", *bots[0]), Bot("p1", *bots[1])))
    ds = duel.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    _upload(ds.environment_state, orc)
    carries = (empty_carry(L, C), empty_carry(L, C))
    ended = 0
    for step in range(200):
        want = orc.duel_step(tuple(b[0] for b in bots), tuple(b[1] for b in bots), carries)
        _, rewards, dones, infos = duel.step(ds)
        torch.cuda.synchronize()
        where = f"persistent duel step {step}"
        _compare_state(ds.environment_state, orc, where)
        for p in range(2):
            _compare_carry(ds.carries[p], carries[p], f"{where} player {p}")
        assert np.array_equal(_np(dones["__all__"]), want["done"]), f"{where}: done"
        assert np.array_equal(_np(infos["winner"]), want["winner"]), f"{where}: winner"
        ended += int(want["done"].sum())
    assert ended >= L, f"only {ended} games ended"
    print(f"persistent duel: {L} games, {ended} ended in 200 steps")


def test_duel_outputs_observations_when_asked():
    """With observations on, the duel's masks and feature maps are those of the carried state."""
    from nanorts_b200.bots import Duel
    from nanorts_b200.env import make
    from oracle.oracle import empty_carry
    from tests.test_gpu_parity import compare_masks

    cfg = BOT_CONFIGS["c4_16x16_both"]
    game = cfg.game(200)
    orc = _oracle_batch(game, [(4, 0), (4, 30)], seed=9)
    L, C = orc.lanes, game.bucket.per_player_capacity
    env = make("NanoRTS", scenario=game, final_observation=False)
    duel = Duel(env, observations=True)
    ds = duel.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    _upload(ds.environment_state, orc)
    carries = (empty_carry(L, C), empty_carry(L, C))
    for step in range(60):
        orc.duel_step((0, 1), (-1, 4), carries)
        duel.step(ds)
        compare_masks(env, ds.environment_state, orc, f"duel step {step}")
        want = orc.observe()
        buf = ds.environment_state._buffers
        for p in range(2):
            assert np.array_equal(_np(buf["feature_maps"][p]), want["feature_maps"][:, p]), f"step {step}: maps {p}"
            assert np.array_equal(_np(buf["scalars"][p]), want["scalars"][:, p]), f"step {step}: scalars {p}"
