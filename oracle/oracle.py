"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs
may import this module.  It is the checker: batches of games live in numpy
arrays with the product's lane-major layout, and every call restates the
reference's JAX program path (see oracle.hpp).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from nanorts_b200 import content as _content
from nanorts_b200.model import (
    PLAYER_COUNT,
    STRATEGY_CODES,
    GameConfig,
    leaf_shapes,
)

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "liboracle.so"
REF_DRAWS = HERE / "_ref" / "libref_draws.so"

LEAVES = (
    "birth", "unit_type", "owner", "cell", "hit_points", "carried_resources", "pending_kind", "pending_direction",
    "pending_none_duration", "pending_target_cell", "pending_produced_type", "pending_issued_at",
    "pending_completes_at", "pending_order", "entity_at", "time", "player_resources", "next_birth",
    "next_pending_order", "alternating_conflict_count", "game_over", "winner", "spawn_overflow",
)


class OracleConfig(ctypes.Structure):
    _fields_ = [
        ("height", ctypes.c_int32), ("width", ctypes.c_int32), ("neutral", ctypes.c_int32),
        ("capacity", ctypes.c_int32), ("types", ctypes.c_int32), ("offsets", ctypes.c_int32),
        ("strategy", ctypes.c_int32), ("max_cycles", ctypes.c_int32),
        ("partial_observability", ctypes.c_int32), ("final_observation", ctypes.c_int32),
        ("terrain", ctypes.c_void_p), ("table", ctypes.c_void_p),
        ("reset", ctypes.c_void_p * len(LEAVES)),
    ]


class OracleStates(ctypes.Structure):
    _fields_ = [
        ("leaf", ctypes.c_void_p * len(LEAVES)),
        ("environment_root", ctypes.c_void_p),
        ("episode_index", ctypes.c_void_p),
    ]


CARRY_FIELDS = ("kind", "unit_birth", "order", "target", "target_birth", "base", "base_birth", "cell", "unit_type")

# family.py:14-17 strategy numbers; unit_types.py:126 TYPE_LIGHT.
WORKER_RUSH, BARRACKS_RUSH = 0, 1
TYPE_LIGHT = 4


class OracleCarry(ctypes.Structure):
    _fields_ = [
        ("field", ctypes.c_void_p * len(CARRY_FIELDS)),
        ("trained", ctypes.c_void_p),
        ("next_order", ctypes.c_void_p),
    ]


def empty_carry(lanes: int, capacity: int) -> dict[str, np.ndarray]:
    """``abstraction.empty_actions`` per lane (abstraction.py:120-135)."""
    carry = {name: np.full((lanes, capacity), -1, np.int32) for name in CARRY_FIELDS}
    carry["trained"] = np.zeros((lanes, capacity), np.uint8)
    carry["next_order"] = np.zeros(lanes, np.int32)
    return carry


def _carry_struct(carry: dict[str, np.ndarray]) -> OracleCarry:
    k = OracleCarry(trained=_ptr(carry["trained"]), next_order=_ptr(carry["next_order"]))
    for f, name in enumerate(CARRY_FIELDS):
        k.field[f] = _ptr(carry[name])
    return k


def astar(free: np.ndarray, start: int, target: int, range_: int) -> tuple[bool, int, int, int]:
    """``pathfinding.search`` (program branch) on a bool[H, W] free-cell grid: (found, step, distance, pops)."""
    free = np.ascontiguousarray(free, np.uint8)
    out = np.zeros(4, np.int32)
    lib().oracle_astar(_ptr(free), free.shape[0], free.shape[1], start, target, range_, _ptr(out))
    return bool(out[0]), int(out[1]), int(out[2]), int(out[3])


def reference_root() -> Path | None:
    """Root of a NanoRTS checkout (the directory holding ``src/nanorts``), or None.

    ``NANORTS_REFERENCE`` names it; without the variable a checkout named
    ``reference`` beside this repository is used when it exists.
    """
    named = os.environ.get("NANORTS_REFERENCE")
    root = Path(named) if named else HERE.parent.parent / "reference"
    return root if (root / "src" / "nanorts").is_dir() else None


def build() -> None:
    """Compile the oracle (and, where a reference checkout exists, its reference builds)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    root = reference_root()
    if root is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"NANORTS_REFERENCE={root}"], check=True)


def _load() -> ctypes.CDLL:
    if not LIBRARY.exists():
        build()
    lib = ctypes.CDLL(str(LIBRARY))
    p = ctypes.c_void_p
    lib.oracle_env_step.argtypes = [p, p, ctypes.c_int64] + [p] * 17 + [ctypes.c_int]
    lib.oracle_core_step.argtypes = [p, p, ctypes.c_int64, p, p, p, p, p, ctypes.c_int]
    lib.oracle_legal_masks.argtypes = [p, p, ctypes.c_int64, p, p, ctypes.c_int]
    lib.oracle_decode_actions.argtypes = [p, p, ctypes.c_int64, p, p, p, ctypes.c_int]
    lib.oracle_visible_cells.argtypes = [p, p, ctypes.c_int64, ctypes.c_int32, p, ctypes.c_int]
    lib.oracle_observe.argtypes = [p, p, ctypes.c_int64, p, p, p, p, ctypes.c_int]
    lib.oracle_reset.argtypes = [p, p, ctypes.c_int64]
    lib.oracle_threefry2x32.argtypes = [ctypes.c_uint32, ctypes.c_uint32, p, p]
    lib.oracle_fold_in.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, p]
    lib.oracle_conflict_draw.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
    lib.oracle_conflict_draw.restype = ctypes.c_int32
    lib.oracle_bot_act.argtypes = [p, p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, p, p, ctypes.c_int]
    lib.oracle_duel_step.argtypes = [p, p, ctypes.c_int64, p, p, p, p] + [p] * 6 + [ctypes.c_int]
    lib.oracle_astar.argtypes = [p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, p]
    lib.oracle_astar.restype = None
    for name in ("oracle_env_step", "oracle_core_step", "oracle_legal_masks", "oracle_observe", "oracle_reset",
                 "oracle_bot_act", "oracle_duel_step", "oracle_decode_actions", "oracle_visible_cells"):
        getattr(lib, name).restype = ctypes.c_int
    return lib


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _load()
    return _LIB


def _ptr(array: np.ndarray) -> int:
    assert array.flags.c_contiguous
    return array.ctypes.data


def reset_state(game: GameConfig) -> dict[str, np.ndarray]:
    """``core.reset``: decide(initial_state) (core/__init__.py:30-32)."""
    return _content.decide(game.initial_state, game.bucket)


class Oracle:
    """Batch of L games stepped by the CPU restatement."""

    def __init__(self, game: GameConfig, lanes: int, *, partial_observability: bool = False,
                 final_observation: bool = False, reward_components: bool = False, threads: int = 0) -> None:
        if game.bucket.index_dtype != np.int16:
            raise ValueError("the oracle handles int16 cell/slot indices only")
        self.game, self.lanes, self.threads = game, lanes, threads
        self.partial = partial_observability
        self.final_observation = final_observation
        self.reward_components = reward_components
        b = game.bucket
        self.capacity, self.cells, self.mask_width = b.per_player_capacity, b.cell_count, b.mask_width
        self._reset = {k: np.ascontiguousarray(v) for k, v in reset_state(game).items()}
        self._terrain = np.ascontiguousarray(game.terrain.reshape(-1).astype(np.uint8))
        self._table = np.ascontiguousarray(game.table)
        self.config = OracleConfig(
            height=b.height, width=b.width, neutral=b.neutral_capacity, capacity=b.per_player_capacity,
            types=b.unit_type_capacity, offsets=b.attack_offset_capacity,
            strategy=STRATEGY_CODES[b.conflict_strategy], max_cycles=game.max_cycles,
            partial_observability=int(partial_observability), final_observation=int(final_observation),
            terrain=_ptr(self._terrain), table=_ptr(self._table),
        )
        for k, name in enumerate(LEAVES):
            self.config.reset[k] = _ptr(self._reset[name])
        shapes = leaf_shapes(b)
        self.state = {name: np.empty((lanes, *shapes[name][0]), shapes[name][1]) for name in LEAVES}
        self.environment_root = np.zeros((lanes, 2), np.uint32)
        self.episode_index = np.zeros(lanes, np.uint32)

    def _states(self) -> OracleStates:
        s = OracleStates(environment_root=_ptr(self.environment_root), episode_index=_ptr(self.episode_index))
        for k, name in enumerate(LEAVES):
            s.leaf[k] = _ptr(self.state[name])
        return s

    def reset(self, keys: np.ndarray) -> dict[str, np.ndarray]:
        """``env.reset`` over lanes (lifecycle.py:44-50); returns the observations."""
        self.environment_root[:] = np.asarray(keys, np.uint32).reshape(self.lanes, 2)
        states = self._states()
        lib().oracle_reset(ctypes.byref(self.config), ctypes.byref(states), self.lanes)
        return self.observe()

    def observe(self) -> dict[str, np.ndarray]:
        fm = [np.empty((self.lanes, self.game.bucket.height, self.game.bucket.width, 6), np.uint8) for _ in range(2)]
        sc = [np.empty((self.lanes, 4), np.int32) for _ in range(2)]
        states = self._states()
        rc = lib().oracle_observe(ctypes.byref(self.config), ctypes.byref(states), self.lanes, _ptr(fm[0]), _ptr(fm[1]),
                                  _ptr(sc[0]), _ptr(sc[1]), self.threads)
        assert rc == 0, rc
        return {"feature_maps": np.stack(fm, 1), "scalars": np.stack(sc, 1)}

    def legal_masks(self) -> np.ndarray:
        """``get_avail_actions``: uint8[L, 2, C, 78] (0/1)."""
        masks = [np.empty((self.lanes, self.capacity, self.mask_width), np.uint8) for _ in range(2)]
        states = self._states()
        rc = lib().oracle_legal_masks(ctypes.byref(self.config), ctypes.byref(states), self.lanes, _ptr(masks[0]),
                                      _ptr(masks[1]), self.threads)
        assert rc == 0, rc
        return np.stack(masks, 1)

    def decode_actions(self, actions: np.ndarray) -> np.ndarray:
        """``decode_actions`` (actions.py:61-84) of int32[L, 2, C, 7] rows: Commands int32[L, 6, 2, C]."""
        actions = np.ascontiguousarray(actions, np.int32)
        a0, a1 = np.ascontiguousarray(actions[:, 0]), np.ascontiguousarray(actions[:, 1])
        commands = np.empty((self.lanes, 6, 2, self.capacity), np.int32)
        states = self._states()
        rc = lib().oracle_decode_actions(ctypes.byref(self.config), ctypes.byref(states), self.lanes, _ptr(a0),
                                         _ptr(a1), _ptr(commands), self.threads)
        assert rc == 0, rc
        return commands

    def visible_cells(self, player: int) -> np.ndarray:
        """Cells ``player`` sees (visibility.py:70-77): bool[L, H, W]."""
        b = self.game.bucket
        out = np.empty((self.lanes, b.height, b.width), np.uint8)
        states = self._states()
        rc = lib().oracle_visible_cells(ctypes.byref(self.config), ctypes.byref(states), self.lanes, player,
                                        _ptr(out), self.threads)
        assert rc == 0, rc
        return out.astype(bool)

    def episode_roots(self) -> np.ndarray:
        """``episode_root`` key data per lane (lifecycle.py:34-37): uint32[L, 2]."""
        out = np.empty((self.lanes, 2), np.uint32)
        for lane in range(self.lanes):
            lib().oracle_fold_in(int(self.environment_root[lane, 0]), int(self.environment_root[lane, 1]),
                                 int(self.episode_index[lane]), out[lane].ctypes.data)
        return out

    def step(self, actions: np.ndarray) -> dict[str, np.ndarray]:
        """The JaxMARL step for actions int32[L, 2, C, 7]."""
        actions = np.ascontiguousarray(actions, np.int32)
        a0, a1 = np.ascontiguousarray(actions[:, 0]), np.ascontiguousarray(actions[:, 1])
        L, b = self.lanes, self.game.bucket
        out = {
            "fm": [np.empty((L, b.height, b.width, 6), np.uint8) for _ in range(2)],
            "sc": [np.empty((L, 4), np.int32) for _ in range(2)],
            "reward": np.empty((L, 2), np.float32),
            "done": np.empty(L, np.uint8),
            "terminated": np.empty(L, np.uint8),
            "truncated": np.empty(L, np.uint8),
            "winner": np.empty(L, np.int32),
            "spawn_overflow": np.empty((L, 2), np.int32),
        }
        final = self.final_observation
        if self.reward_components:
            out["reward_components"] = np.empty((L, 2, 6), np.float32)
        if final:
            out["final_fm"] = [np.empty((L, b.height, b.width, 6), np.uint8) for _ in range(2)]
            out["final_sc"] = [np.empty((L, 4), np.int32) for _ in range(2)]
        states = self._states()
        rc = lib().oracle_env_step(
            ctypes.byref(self.config), ctypes.byref(states), L, _ptr(a0), _ptr(a1),
            _ptr(out["fm"][0]), _ptr(out["fm"][1]), _ptr(out["sc"][0]), _ptr(out["sc"][1]), _ptr(out["reward"]),
            _ptr(out["done"]), _ptr(out["terminated"]), _ptr(out["truncated"]), _ptr(out["winner"]),
            _ptr(out["spawn_overflow"]),
            _ptr(out["final_fm"][0]) if final else None, _ptr(out["final_fm"][1]) if final else None,
            _ptr(out["final_sc"][0]) if final else None, _ptr(out["final_sc"][1]) if final else None,
            _ptr(out["reward_components"]) if self.reward_components else None,
            self.threads,
        )
        assert rc == 0, rc
        result = {
            "feature_maps": np.stack(out["fm"], 1),
            "scalars": np.stack(out["sc"], 1),
            "reward": out["reward"],
            "done": out["done"].astype(bool),
            "terminated": out["terminated"].astype(bool),
            "truncated": out["truncated"].astype(bool),
            "winner": out["winner"],
            "spawn_overflow": out["spawn_overflow"],
        }
        if self.reward_components:
            result["reward_components"] = out["reward_components"]
        if final:
            result["final_feature_maps"] = np.stack(out["final_fm"], 1)
            result["final_scalars"] = np.stack(out["final_sc"], 1)
        return result

    def core_step(self, commands: np.ndarray, keys: np.ndarray) -> dict[str, np.ndarray]:
        """``core.step`` with explicit Commands int32[L, 6, 2, C] and keys uint32[L, 2]."""
        commands = np.ascontiguousarray(commands, np.int32)
        keys = np.ascontiguousarray(keys, np.uint32)
        L = self.lanes
        terminated, truncated = np.empty(L, np.uint8), np.empty(L, np.uint8)
        reward = np.empty((L, 2), np.float32)
        states = self._states()
        rc = lib().oracle_core_step(ctypes.byref(self.config), ctypes.byref(states), L, _ptr(commands), _ptr(keys),
                                    _ptr(terminated), _ptr(truncated), _ptr(reward), self.threads)
        assert rc == 0, rc
        return {"terminated": terminated.astype(bool), "truncated": truncated.astype(bool), "reward": reward}

    def bot_act(self, player: int, strategy: int, trained: int, carry: dict[str, np.ndarray]) -> np.ndarray:
        """``family.act`` for one player's rush bot; updates ``carry`` in place, returns Commands int32[L, 6, 2, C]."""
        commands = np.empty((self.lanes, 6, 2, self.capacity), np.int32)
        k = _carry_struct(carry)
        states = self._states()
        rc = lib().oracle_bot_act(ctypes.byref(self.config), ctypes.byref(states), self.lanes, player, strategy,
                                  trained, ctypes.byref(k), _ptr(commands), self.threads)
        assert rc == 0, rc
        return commands

    def duel_step(self, strategies: tuple[int, int], trained: tuple[int, int],
                  carries: tuple[dict[str, np.ndarray], dict[str, np.ndarray]]) -> dict[str, np.ndarray]:
        """Bot against bot: both players' rush bots act, core.step, auto-reset (carries too)."""
        L = self.lanes
        st = np.ascontiguousarray(strategies, np.int32)
        tr = np.ascontiguousarray(trained, np.int32)
        out = {
            "reward": np.empty((L, 2), np.float32), "done": np.empty(L, np.uint8),
            "terminated": np.empty(L, np.uint8), "truncated": np.empty(L, np.uint8),
            "winner": np.empty(L, np.int32), "spawn_overflow": np.empty((L, 2), np.int32),
        }
        k0, k1 = _carry_struct(carries[0]), _carry_struct(carries[1])
        states = self._states()
        rc = lib().oracle_duel_step(ctypes.byref(self.config), ctypes.byref(states), L, _ptr(st), _ptr(tr),
                                    ctypes.byref(k0), ctypes.byref(k1), _ptr(out["reward"]), _ptr(out["done"]),
                                    _ptr(out["terminated"]), _ptr(out["truncated"]), _ptr(out["winner"]),
                                    _ptr(out["spawn_overflow"]), self.threads)
        assert rc == 0, rc
        for name in ("done", "terminated", "truncated"):
            out[name] = out[name].astype(bool)
        return out


def sample_uniform_legal(masks: np.ndarray, widths: tuple[int, ...], rng: np.random.Generator) -> np.ndarray:
    """Draw one legal value per factor, uniformly over the factor's set mask bits (0 when none).

    masks: uint8[..., 78] -> int32[..., 7].  The host-side stand-in for the
    reference benchmark's per-factor ``jax.random.categorical`` over masked
    logits (README.md:53-63), which draws each legal value with equal chance.
    """
    bounds = np.cumsum((0, *widths))
    shape = masks.shape[:-1]
    out = np.zeros((*shape, len(widths)), np.int32)
    for f, (lo, hi) in enumerate(zip(bounds[:-1], bounds[1:])):
        group = masks[..., lo:hi].astype(bool)
        count = group.sum(-1)
        pick = np.floor(rng.random(shape) * np.maximum(count, 1)).astype(np.int64)
        # index of the pick-th set bit
        csum = np.cumsum(group, -1)
        chosen = np.argmax(csum > pick[..., None], -1)
        out[..., f] = np.where(count > 0, chosen, 0)
    return out


def ref_draws() -> ctypes.CDLL | None:
    """The reference's conflict_draw.cuh built as host code, when it was built here."""
    if not REF_DRAWS.exists():
        return None
    ref = ctypes.CDLL(str(REF_DRAWS))
    p = ctypes.c_void_p
    ref.ref_threefry2x32.argtypes = [ctypes.c_uint32, ctypes.c_uint32, p, p]
    ref.ref_fold_in.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, p]
    ref.ref_conflict_draw.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
    ref.ref_conflict_draw.restype = ctypes.c_int32
    return ref


PLAYERS = PLAYER_COUNT
