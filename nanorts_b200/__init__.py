"""nanorts_b200: NanoRTS's batched environment step, native to B200 (sm_100a).

Public surface (the reference's JaxMARL entry points, src/nanorts/__init__.py
and src/nanorts/adapters/jaxmarl/__init__.py): ``make``,
``map_name_to_scenario``, ``scenario_names``, ``load_game``.
"""

from nanorts_b200.content import (
    CAPACITY_PROFILES,
    load_game,
    map_name_to_scenario,
    scenario_names,
    with_unit_type_table,
)
from nanorts_b200.model import ConflictStrategy, GameConfig, ModelError, UnitTypeTableVersion


def make(env_id: str, **options):
    """``nanorts.make`` (adapters/jaxmarl/facade.py:43-56); see nanorts_b200.env.make."""
    from nanorts_b200.env import make as _make

    return _make(env_id, **options)


__all__ = [
    "CAPACITY_PROFILES",
    "ConflictStrategy",
    "GameConfig",
    "ModelError",
    "UnitTypeTableVersion",
    "load_game",
    "make",
    "map_name_to_scenario",
    "scenario_names",
    "with_unit_type_table",
]
