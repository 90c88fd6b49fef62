"""Rush-family scripted bots (WorkerRush, LightRush) on the sm_100a kernels.

Mirrors the reference's bot interface (src/nanorts/bots/bot.py:13-22): a
``Bot`` has a ``name``, an ``init`` giving the empty carry (AbstractActions,
bots/abstraction.py:70-135) and an ``act`` that turns (carry, state, player)
into Commands (bots/family.py:34-69).  Carries and Commands are batched like
the environment: every tensor has a leading lane axis ``L``.

``Duel`` steps games where both players are bots (player 0 and player 1 each
pick Commands from the step's starting state, bots/seat.py:152-157), in one
kernel launch per step: both bots, the core step, the outcome and the
auto-reset of the state and of both carries.

The bots ignore their keys (bots/worker_rush.py:13-15, bots/light_rush.py:13-18)
and CANCEL_BOTH draws nothing, so the games of a Duel from one scenario stay
identical lane to lane unless their states differ.
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Any

import torch

from nanorts_b200.env import ALL_AGENTS, AGENTS, EnvironmentState, NanoRTS, Telemetry, _ptr
from nanorts_b200.model import PLAYER_COUNT, TYPE_LIGHT, ModelError
from nanorts_b200.runtime import BotSpec, Outputs, check, library

WORKER_RUSH, BARRACKS_RUSH = 0, 1  # bots/family.py:14-15
CARRY_FIELDS = ("kind", "unit_birth", "order", "target", "target_birth", "base", "base_birth", "cell", "unit_type")
COMMAND_FIELDS = ("kind", "direction", "none_duration", "target_cell", "produced_type", "request_order")


@dataclasses.dataclass
class AbstractActions:
    """A rush bot's carry over L lanes (bots/abstraction.py:70-81)."""

    kind: torch.Tensor          # int32 [L, C]
    unit_birth: torch.Tensor
    order: torch.Tensor
    target: torch.Tensor
    target_birth: torch.Tensor
    base: torch.Tensor
    base_birth: torch.Tensor
    cell: torch.Tensor
    unit_type: torch.Tensor
    trained: torch.Tensor       # uint8 [L, C] (0/1)
    next_order: torch.Tensor    # int32 [L]

    def fields(self) -> list[torch.Tensor]:
        return [getattr(self, name) for name in CARRY_FIELDS]

    def reset_where(self, done: torch.Tensor) -> None:
        """Back to empty_actions on the lanes where ``done`` (bots/seat.py:127)."""
        mask = done.to(torch.bool)
        for t in self.fields():
            t[mask] = -1
        self.trained[mask] = 0
        self.next_order[mask] = 0


def empty_actions(lanes: int, capacity: int, device: Any) -> AbstractActions:
    """``abstraction.empty_actions`` for L lanes (bots/abstraction.py:120-135)."""
    fields = {name: torch.full((lanes, capacity), -1, dtype=torch.int32, device=device) for name in CARRY_FIELDS}
    return AbstractActions(**fields, trained=torch.zeros((lanes, capacity), dtype=torch.uint8, device=device),
                           next_order=torch.zeros((lanes,), dtype=torch.int32, device=device))


def _spec(strategy: int, trained: int, carry: AbstractActions) -> BotSpec:
    spec = BotSpec(strategy=strategy, trained=trained)
    for f, t in enumerate(carry.fields()):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ModelError("carry fields must be contiguous int32 tensors")
        spec.carry.field[f] = t.data_ptr()
    spec.carry.trained = _ptr(carry.trained)
    spec.carry.next_order = _ptr(carry.next_order)
    return spec


@dataclasses.dataclass(frozen=True)
class Bot:
    """A scripted player (bots/bot.py:13-22) of the rush family."""

    name: str
    strategy: int
    trained: int = -1

    def init(self, env: NanoRTS, lanes: int) -> AbstractActions:
        return empty_actions(lanes, env.game.bucket.per_player_capacity, env.device)

    def act(self, key: Any, carry: AbstractActions, state: EnvironmentState, env: NanoRTS, player: int) -> torch.Tensor:
        """family.act: updates ``carry`` in place; returns Commands int32 [L, 6, 2, C]
        (fields kind, direction, none_duration, target_cell, produced_type, request_order).
        The key is ignored, as by the reference's rush bots."""
        del key
        if player not in (0, 1):
            raise ModelError(f"player must be 0 or 1, not {player!r}")
        L, C = state.lanes, env.game.bucket.per_player_capacity
        commands = torch.empty((L, len(COMMAND_FIELDS), PLAYER_COUNT, C), dtype=torch.int32, device=env.device)
        spec = _spec(self.strategy, self.trained, carry)
        ptrs = env._state_ptrs(state)
        check(library().nrts_bot_act(ctypes.byref(env._extents), ctypes.byref(env._content), ctypes.byref(ptrs), L,
                                     player, ctypes.byref(spec), _ptr(commands), env._stream()))
        return commands


workerRushAI = Bot("workerRushAI", WORKER_RUSH)                # bots/worker_rush.py:13-20
lightRushAI = Bot("lightRushAI", BARRACKS_RUSH, TYPE_LIGHT)    # bots/light_rush.py:13-23
ROSTER = {bot.name: bot for bot in (workerRushAI, lightRushAI)}


@dataclasses.dataclass
class DuelState:
    environment_state: EnvironmentState
    carries: tuple[AbstractActions, AbstractActions]


class Duel:
    """Bot against bot over one NanoRTS environment (one launch per step)."""

    def __init__(self, env: NanoRTS, bots: tuple[Bot, Bot] = (workerRushAI, lightRushAI), *,
                 observations: bool = False) -> None:
        self.env = env
        self.bots = tuple(bots)
        self.observations = observations
        if len(self.bots) != PLAYER_COUNT:
            raise ModelError("a Duel needs one bot per player")

    def reset(self, key: torch.Tensor) -> DuelState:
        _, state = self.env.reset(key)
        carries = tuple(bot.init(self.env, state.lanes) for bot in self.bots)
        return DuelState(environment_state=state, carries=carries)  # type: ignore[arg-type]

    def step(self, duel: DuelState) -> tuple[DuelState, dict, dict, dict]:
        """One step of every game; returns (state, rewards, dones, infos) like env.step without observations."""
        env, state = self.env, duel.environment_state
        buf = env._buffers(state)
        out = Outputs()
        for name in ("reward", "done", "terminated", "truncated", "winner", "spawn_overflow"):
            setattr(out, name, _ptr(buf[name]))
        if self.observations:
            for p in range(PLAYER_COUNT):
                out.masks[p] = _ptr(buf["masks"][p])
                out.feature_maps[p] = _ptr(buf["feature_maps"][p])
                out.scalars[p] = _ptr(buf["scalars"][p])
        out.reverse_order = state._launches & 1
        state._launches += 1
        specs = (BotSpec * PLAYER_COUNT)(*(_spec(b.strategy, b.trained, c) for b, c in zip(self.bots, duel.carries)))
        ptrs = env._state_ptrs(state)
        check(library().nrts_duel_step(ctypes.byref(env._extents), ctypes.byref(env._content), ctypes.byref(ptrs),
                                       state.lanes, specs, ctypes.byref(out), env._stream()))
        state._masks_current = self.observations
        done = buf["done"].view(torch.bool)
        rewards = {agent: buf["reward"][:, p] for p, agent in enumerate(AGENTS)}
        dones = {agent: done for agent in AGENTS} | {ALL_AGENTS: done}
        infos = {
            "terminated": buf["terminated"].view(torch.bool),
            "truncated": buf["truncated"].view(torch.bool),
            "winner": buf["winner"],
            "telemetry": Telemetry(spawn_overflow=buf["spawn_overflow"]),
        }
        return duel, rewards, dones, infos
