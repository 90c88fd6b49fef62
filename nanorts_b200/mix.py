"""GroupMix: several groups of NanoRTS games stepped as one batch of rows.

Mirrors the reference's ``GroupMix`` (src/nanorts/bots/mix.py:16-260): each
``Group`` is an environment and a lane count; the mix publishes rows in
agent-major order per group (a group of L lanes owns 2L consecutive rows,
player_0's L then player_1's L), resets from one array of roots split by
group, and steps from one array of action rows.  Groups whose games share
their extents (the reference's bucket, bots/mix.py:130-139) step in ONE
launch (``nrts_step_groups``, the counterpart of ``core.step_groups``), and
the kernel writes masks, feature maps and scalars straight into the mix's
row buffers: no concatenation copies on the device.

The reference refuses groups whose rows differ (``_refuse_unlike_rows``):
equal observation and action spaces and equal ``final_observation`` and
``reward_components`` flags; so does this mix.
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Any

import torch

from nanorts_b200.env import EnvironmentState, NanoRTS, SymbolicObservation, Telemetry, _ptr
from nanorts_b200.model import PLAYER_COUNT, ModelError
from nanorts_b200.runtime import MAX_GROUPS, GroupStep, Outputs, check, library


@dataclasses.dataclass(frozen=True)
class Group:
    environment: NanoRTS
    lanes: int


def _row_signature(env: NanoRTS) -> tuple:
    b = env.game.bucket
    return (b.height, b.width, b.per_player_capacity, env.layout.mask_width, env.layout.mask_form,
            env.layout.feature_maps_dtype, env.final_observation, env.reward_components, env.device)


def _launch_key(env: NanoRTS) -> tuple:
    x = env._extents
    return (x.height, x.width, x.neutral, x.capacity, x.types, x.offsets, x.strategy, x.partial_observability)


class GroupMix:
    """Groups of games as one batch of agent-major rows (bots/mix.py:16-101)."""

    def __init__(self, groups: list[Group] | tuple[Group, ...]) -> None:
        self.groups = tuple(groups)
        if not self.groups:
            raise ModelError("GroupMix refuses an empty group list")
        for index, group in enumerate(self.groups):
            if not isinstance(group.lanes, int) or group.lanes < 1:
                raise ModelError(f"GroupMix refuses group {index}: lanes={group.lanes!r} is not a positive int")
        first = _row_signature(self.groups[0].environment)
        for index, group in enumerate(self.groups[1:], start=1):
            if _row_signature(group.environment) != first:
                raise ModelError(f"GroupMix refuses group {index}: its rows are not group 0's - the groups' "
                                 "environments must publish equal observation and action spaces and equal infos")
        # Launches: groups that share their extents, at most MAX_GROUPS per launch.
        by_key: dict[tuple, list[int]] = {}
        for index, group in enumerate(self.groups):
            by_key.setdefault(_launch_key(group.environment), []).append(index)
        self.launches = [members[i:i + MAX_GROUPS] for members in by_key.values()
                         for i in range(0, len(members), MAX_GROUPS)]
        self._buffers: dict[str, torch.Tensor] | None = None

    @property
    def lanes(self) -> int:
        return sum(group.lanes for group in self.groups)

    @property
    def rows(self) -> int:
        return sum(PLAYER_COUNT * group.lanes for group in self.groups)

    def _row_counts(self) -> list[int]:
        return [PLAYER_COUNT * group.lanes for group in self.groups]

    def slices(self) -> tuple[slice, ...]:
        """Each group's rows (bots/mix.py:41-42)."""
        out, start = [], 0
        for count in self._row_counts():
            out.append(slice(start, start + count))
            start += count
        return tuple(out)

    # -- row buffers ------------------------------------------------------------
    def _allocate(self) -> dict[str, torch.Tensor]:
        if self._buffers is not None:
            return self._buffers
        env = self.groups[0].environment
        b, dev, R = env.game.bucket, env.device, self.rows
        C = b.per_player_capacity
        buf = {
            "feature_maps": torch.empty((R, b.height, b.width, 6), dtype=torch.uint8, device=dev),
            "scalars": torch.empty((R, 4), dtype=torch.int32, device=dev),
        }
        if env.layout.mask_form == "packed":
            buf["packed_masks"] = torch.empty((R, C, 3), dtype=torch.uint32, device=dev)
        else:
            buf["masks"] = torch.empty((R, C, env.layout.mask_width), dtype=torch.uint8, device=dev)
        if env.final_observation:
            buf["final_feature_maps"] = torch.empty_like(buf["feature_maps"])
            buf["final_scalars"] = torch.empty_like(buf["scalars"])
        self._buffers = buf
        return buf

    def _row_ptrs(self, name: str, start: int, lanes: int) -> tuple[int, int]:
        t = self._buffers[name]
        return _ptr(t[start]), _ptr(t[start + lanes])

    def _observations(self, prefix: str = "") -> SymbolicObservation:
        buf = self._buffers
        return SymbolicObservation(feature_maps=buf[prefix + "feature_maps"], scalars=buf[prefix + "scalars"])

    # -- the reference's surface ------------------------------------------------
    def reset(self, roots: torch.Tensor) -> tuple[SymbolicObservation, tuple[EnvironmentState, ...]]:
        """bots/mix.py:45-56: roots uint32 [lanes, 2] split by group; observations as rows."""
        roots = torch.as_tensor(roots)
        if roots.shape != (self.lanes, 2):
            raise ModelError(f"GroupMix.reset expects roots [{self.lanes}, 2], not {tuple(roots.shape)}")
        buf = self._allocate()
        states, lane, row = [], 0, 0
        for group in self.groups:
            env, L = group.environment, group.lanes
            keys = roots[lane:lane + L].to(device=env.device, dtype=torch.uint32).contiguous()
            state = env._empty_state(L)
            env._buffers(state)
            out = Outputs()
            name = "packed_masks" if env.packed else "masks"
            target = out.packed_masks if env.packed else out.masks
            target[0], target[1] = self._row_ptrs(name, row, L)
            out.feature_maps[0], out.feature_maps[1] = self._row_ptrs("feature_maps", row, L)
            out.scalars[0], out.scalars[1] = self._row_ptrs("scalars", row, L)
            ptrs = env._state_ptrs(state)
            check(library().nrts_reset(ctypes.byref(env._extents), ctypes.byref(env._content), ctypes.byref(ptrs), L,
                                       _ptr(keys), ctypes.byref(out), env._stream()))
            states.append(state)
            lane += L
            row += PLAYER_COUNT * L
        return self._observations(), tuple(states)

    def step(self, key: Any, states: tuple[EnvironmentState, ...], actions: torch.Tensor
             ) -> tuple[SymbolicObservation, tuple[EnvironmentState, ...], torch.Tensor, torch.Tensor, dict]:
        """bots/mix.py:58-73: action rows int32 [rows, C, 7]; returns rows of
        observations, the states, rewards [rows], dones [rows] and infos."""
        del key
        buf = self._allocate()
        env0 = self.groups[0].environment
        C = env0.game.bucket.per_player_capacity
        if actions.shape != (self.rows, C, 7) or actions.dtype != torch.int32 or not actions.is_contiguous():
            raise ModelError(f"GroupMix.step expects contiguous int32 action rows [{self.rows}, {C}, 7]")
        if len(states) != len(self.groups):
            raise ModelError("GroupMix.step expects one state per group")
        starts = [s.start for s in self.slices()]
        keep: list[Any] = []
        for members in self.launches:
            table = (GroupStep * len(members))()
            for j, index in enumerate(members):
                group, state = self.groups[index], states[index]
                env, L, row = group.environment, group.lanes, starts[index]
                gbuf = env._buffers(state)
                out = Outputs()
                name = "packed_masks" if env.packed else "masks"
                target = out.packed_masks if env.packed else out.masks
                target[0], target[1] = self._row_ptrs(name, row, L)
                out.feature_maps[0], out.feature_maps[1] = self._row_ptrs("feature_maps", row, L)
                out.scalars[0], out.scalars[1] = self._row_ptrs("scalars", row, L)
                if env.final_observation:
                    out.final_feature_maps[0], out.final_feature_maps[1] = self._row_ptrs("final_feature_maps", row, L)
                    out.final_scalars[0], out.final_scalars[1] = self._row_ptrs("final_scalars", row, L)
                for field in ("reward", "done", "terminated", "truncated", "winner", "spawn_overflow"):
                    setattr(out, field, _ptr(gbuf[field]))
                if env.reward_components:
                    out.reward_components = _ptr(gbuf["reward_components"])
                out.reverse_order = state._launches & 1
                state._launches += 1
                ptrs = env._state_ptrs(state)
                keep.extend((out, ptrs))
                table[j].extents = ctypes.addressof(env._extents)
                table[j].content = ctypes.addressof(env._content)
                table[j].state = ctypes.addressof(ptrs)
                table[j].lanes = L
                table[j].actions[0] = _ptr(actions[row])
                table[j].actions[1] = _ptr(actions[row + L])
                table[j].outputs = ctypes.addressof(out)
                state._masks_current = False  # the masks of this state live in the mix's rows
            check(library().nrts_step_groups(table, len(members), env0._stream()))
        # Per-game outputs to agent-major rows (bots/mix.py:198-224).
        rewards, dones, infos_parts = [], [], {"terminated": [], "truncated": [], "winner": [], "spawn_overflow": [],
                                               "reward_components": []}
        for group, state in zip(self.groups, states):
            gbuf = group.environment._buffers(state)
            rewards.append(gbuf["reward"].t().reshape(-1))
            done = gbuf["done"].view(torch.bool)
            dones.append(done.repeat(PLAYER_COUNT))
            for name in ("terminated", "truncated"):
                infos_parts[name].append(gbuf[name].view(torch.bool).repeat(PLAYER_COUNT))
            infos_parts["winner"].append(gbuf["winner"].repeat(PLAYER_COUNT))
            infos_parts["spawn_overflow"].append(gbuf["spawn_overflow"].repeat(PLAYER_COUNT, 1))
            if group.environment.reward_components:
                infos_parts["reward_components"].append(gbuf["reward_components"].transpose(0, 1).reshape(-1, 6))
        infos: dict[str, Any] = {
            "terminated": torch.cat(infos_parts["terminated"]),
            "truncated": torch.cat(infos_parts["truncated"]),
            "winner": torch.cat(infos_parts["winner"]),
            "telemetry": Telemetry(spawn_overflow=torch.cat(infos_parts["spawn_overflow"])),
        }
        if env0.final_observation:
            infos["final_observation"] = self._observations("final_")
        if infos_parts["reward_components"]:
            infos["reward_components"] = torch.cat(infos_parts["reward_components"])
        return self._observations(), states, torch.cat(rewards), torch.cat(dones), infos

    def get_avail_actions(self, states: tuple[EnvironmentState, ...]) -> torch.Tensor:
        """bots/mix.py:75-82: the rows the last reset or step wrote."""
        buf = self._allocate()
        if "packed_masks" in buf:
            return buf["packed_masks"]
        return buf["masks"].view(torch.bool)

    def get_slot_cells(self, states: tuple[EnvironmentState, ...]) -> torch.Tensor:
        """bots/mix.py:84-91: int32 [rows, C]."""
        parts = []
        for group, state in zip(self.groups, states):
            cells = group.environment.get_slot_cells(state)
            parts.extend([cells["player_0"], cells["player_1"]])
        return torch.cat(parts)
