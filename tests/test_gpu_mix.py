"""GroupMix on the sm_100a path vs per-group CPU oracles (needs a B200).

Three groups of 16x16 games with different maps, unit tables, time limits
and observability: the first two share their extents and step in one
nrts_step_groups launch, the third (partial observability) in its own.  Rows
are agent-major per group, as bots/mix.py publishes them.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion
from tests.parity import random_keys, sample
from tests.test_gpu_parity import compare_state

pytestmark = pytest.mark.gpu

GROUPS = (
    ("basesWorkers16x16A", UnitTypeTableVersion.ORIGINAL, 150, False, 20),
    ("basesWorkers16x16B", UnitTypeTableVersion.ORIGINAL_FINETUNED, 90, False, 13),
    ("basesWorkers16x16C", UnitTypeTableVersion.ORIGINAL, 120, True, 9),
)


def _agent_rows(per_player: np.ndarray) -> np.ndarray:
    """[L, 2, ...] -> [2L, ...] agent-major."""
    return np.concatenate([per_player[:, 0], per_player[:, 1]])


def test_group_mix_matches_per_group_oracles():
    from nanorts_b200.content import map_name_to_scenario
    from nanorts_b200.env import make
    from nanorts_b200.mix import Group, GroupMix
    from oracle.oracle import Oracle

    envs, oracles, games = [], [], []
    for name, utt, max_cycles, partial, lanes in GROUPS:
        game = map_name_to_scenario(name, utt=utt, conflict_strategy=ConflictStrategy.CANCEL_RANDOM,
                                    max_cycles=max_cycles)
        games.append(game)
        envs.append(make("NanoRTS", scenario=game, partial_observability=partial, final_observation=True,
                         reward_components=True))
        oracles.append(Oracle(game, lanes, partial_observability=partial, final_observation=True,
                              reward_components=True))
    mix = GroupMix([Group(env, lanes) for env, (*_, lanes) in zip(envs, GROUPS)])
    assert [len(launch) for launch in mix.launches] == [2, 1]
    rng = np.random.default_rng(17)
    roots = random_keys(rng, mix.lanes)
    obs, states = mix.reset(torch.from_numpy(roots.view(np.int32)).cuda().view(torch.uint32))
    start = 0
    want_obs = []
    for orc, (*_, lanes) in zip(oracles, GROUPS):
        want_obs.append(orc.reset(roots[start:start + lanes]))
        start += lanes
    assert np.array_equal(obs.feature_maps.cpu().numpy(),
                          np.concatenate([_agent_rows(w["feature_maps"]) for w in want_obs]))
    episodes = 0
    for t in range(260):
        masks = mix.get_avail_actions(states).cpu().numpy().astype(np.uint8)
        want_masks = np.concatenate([_agent_rows(orc.legal_masks()) for orc in oracles])
        assert np.array_equal(masks, want_masks), f"step {t}: mask rows"
        actions, wants = [], []
        for orc in oracles:
            a = sample(orc.legal_masks(), rng, 0.3)
            actions.append(_agent_rows(a))
            wants.append(orc.step(a))
        rows = torch.from_numpy(np.ascontiguousarray(np.concatenate(actions))).cuda()
        obs, states, rewards, dones, infos = mix.step(None, states, rows)
        where = f"step {t}"
        for k, (state, orc) in enumerate(zip(states, oracles)):
            compare_state(state, orc, f"{where} group {k}")
        cat = lambda name: np.concatenate([_agent_rows(w[name]) for w in wants])  # noqa: E731
        assert np.array_equal(obs.feature_maps.cpu().numpy(), cat("feature_maps")), f"{where}: feature maps"
        assert np.array_equal(obs.scalars.cpu().numpy(), cat("scalars")), f"{where}: scalars"
        assert np.array_equal(infos["final_observation"].feature_maps.cpu().numpy(), cat("final_feature_maps"))
        assert np.array_equal(rewards.cpu().numpy(), cat("reward")), f"{where}: rewards"
        assert np.array_equal(infos["reward_components"].cpu().numpy(), cat("reward_components")), f"{where}: components"
        done_rows = np.concatenate([np.concatenate([w["done"], w["done"]]) for w in wants])
        assert np.array_equal(dones.cpu().numpy(), done_rows), f"{where}: dones"
        winner_rows = np.concatenate([np.concatenate([w["winner"], w["winner"]]) for w in wants])
        assert np.array_equal(infos["winner"].cpu().numpy(), winner_rows), f"{where}: winner"
        episodes += int(sum(w["done"].sum() for w in wants))
    assert episodes > 0
    cells = mix.get_slot_cells(states).cpu().numpy()
    assert cells.shape == (mix.rows, games[0].bucket.per_player_capacity)
