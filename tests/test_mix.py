"""GroupMix host logic on CPU: row slices, launch grouping, refusals
(bots/mix.py:16-43, :126-139, :227-240)."""

from __future__ import annotations

import pytest

from nanorts_b200.content import map_name_to_scenario
from nanorts_b200.model import ConflictStrategy, ModelError, UnitTypeTableVersion


def _env(name="basesWorkers16x16A", *, strategy=ConflictStrategy.CANCEL_RANDOM, partial=False, final=True,
         utt=UnitTypeTableVersion.ORIGINAL):
    from nanorts_b200.env import make

    game = map_name_to_scenario(name, utt=utt, conflict_strategy=strategy)
    return make("NanoRTS", scenario=game, partial_observability=partial, final_observation=final, device="cpu")


def test_rows_slices_and_shared_launches():
    from nanorts_b200.mix import Group, GroupMix

    a, b = _env(), _env("basesWorkers16x16B", utt=UnitTypeTableVersion.ORIGINAL_FINETUNED)
    c = _env("basesWorkers16x16C", strategy=ConflictStrategy.CANCEL_BOTH)
    mix = GroupMix([Group(a, 5), Group(b, 3), Group(c, 4)])
    assert mix.lanes == 12 and mix.rows == 24
    assert mix.slices() == (slice(0, 10), slice(10, 16), slice(16, 24))
    assert mix.launches == [[0, 1], [2]]  # a and b share their extents; c's conflict strategy differs


def test_at_most_eight_groups_per_launch():
    from nanorts_b200.mix import Group, GroupMix

    env = _env()
    mix = GroupMix([Group(env, 1) for _ in range(11)])
    assert [len(m) for m in mix.launches] == [8, 3]


def test_unlike_rows_and_bad_lanes_are_refused():
    from nanorts_b200.mix import Group, GroupMix

    with pytest.raises(ModelError):
        GroupMix([])
    with pytest.raises(ModelError):
        GroupMix([Group(_env(), 0)])
    with pytest.raises(ModelError):  # 8x8 rows are not 16x16 rows
        GroupMix([Group(_env(), 2), Group(_env("basesWorkers8x8"), 2)])
    with pytest.raises(ModelError):  # final_observation differs
        GroupMix([Group(_env(), 2), Group(_env(final=False), 2)])
