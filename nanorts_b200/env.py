"""The NanoRTS JaxMARL surface over the sm_100a kernels.

Mirrors ``src/nanorts/adapters/jaxmarl/facade.py`` (``make`` and ``NanoRTS``
with ``reset``, ``step``, ``get_avail_actions``, ``get_obs``,
``get_slot_cells``, ``layout``) for a batch of games held in torch tensors on
one CUDA device.  The reference environment is written per game and batched
by ``jax.vmap``; this one is batched natively: every leaf has a leading lane
axis ``L``, the same layout ``vmap`` gives the reference's pytrees.

Differences a caller of the reference sees:
  * keys are threefry key data, ``uint32[L, 2]`` tensors (``jax.random.key_data``
    of the per-game keys);
  * ``step`` updates the EnvironmentState in place (the reference's kernel
    path aliases the state buffers too) and returns the same object;
  * outputs of a call are views of per-state buffers that the next call on
    that state overwrites; ``.clone()`` what must be kept.
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Any

import numpy as np
import torch

from nanorts_b200 import content as _content
from nanorts_b200.model import (
    ACTION_KIND_COUNT,
    DIRECTION_COUNT,
    KIND_NONE,
    PLAYER_COUNT,
    STRATEGY_CODES,
    GameConfig,
    ModelError,
    UnitTypeTableVersion,
    leaf_shapes,
)
from nanorts_b200.runtime import Content, Extents, Outputs, StatePtrs, check, check_device, library

AGENTS = tuple(f"player_{p}" for p in range(PLAYER_COUNT))
ALL_AGENTS = "__all__"
ENVIRONMENT_IDS = ("NanoRTS",)
ACTION_FACTORS = ("kind", "move_direction", "harvest_direction", "return_direction", "produce_direction",
                  "produce_type", "attack_offset")
MASK_FORMS = ("rows", "packed")  # adapters/factors.py:23
MASK_WORDS = 3
NONE_DURATION = 1

LEAVES = (
    "birth", "unit_type", "owner", "cell", "hit_points", "carried_resources", "pending_kind", "pending_direction",
    "pending_none_duration", "pending_target_cell", "pending_produced_type", "pending_issued_at",
    "pending_completes_at", "pending_order", "entity_at", "time", "player_resources", "next_birth",
    "next_pending_order", "alternating_conflict_count", "game_over", "winner", "spawn_overflow",
)

_TORCH_DTYPES = {
    np.dtype(np.int8): torch.int8, np.dtype(np.int16): torch.int16, np.dtype(np.int32): torch.int32,
    np.dtype(np.bool_): torch.bool, np.dtype(np.uint8): torch.uint8,
}


@dataclasses.dataclass
class Telemetry:
    spawn_overflow: torch.Tensor


@dataclasses.dataclass
class State:
    """Core State of L games, one tensor per reference leaf (model/state.py:35-80)."""

    birth: torch.Tensor
    unit_type: torch.Tensor
    owner: torch.Tensor
    cell: torch.Tensor
    hit_points: torch.Tensor
    carried_resources: torch.Tensor
    pending_kind: torch.Tensor
    pending_direction: torch.Tensor
    pending_none_duration: torch.Tensor
    pending_target_cell: torch.Tensor
    pending_produced_type: torch.Tensor
    pending_issued_at: torch.Tensor
    pending_completes_at: torch.Tensor
    pending_order: torch.Tensor
    entity_at: torch.Tensor
    time: torch.Tensor
    player_resources: torch.Tensor
    next_birth: torch.Tensor
    next_pending_order: torch.Tensor
    alternating_conflict_count: torch.Tensor
    game_over: torch.Tensor
    winner: torch.Tensor
    spawn_overflow: torch.Tensor

    @property
    def active(self) -> torch.Tensor:
        return self.birth != -1

    @property
    def telemetry(self) -> Telemetry:
        return Telemetry(spawn_overflow=self.spawn_overflow)

    def leaves(self) -> list[torch.Tensor]:
        return [getattr(self, name) for name in LEAVES]


class StepInfos(dict):
    """The step's infos; values are views of the state's output buffers that
    the next step on the same state overwrites.  ``spawn_overflowed`` is
    derived from the telemetry when first read after a step."""

    def __init__(self, spawn_overflow: torch.Tensor) -> None:
        super().__init__()
        self._spawn_overflow = spawn_overflow

    def stale(self) -> None:
        super().pop("spawn_overflowed", None)

    def _derive(self) -> None:
        if not super().__contains__("spawn_overflowed"):
            super().__setitem__("spawn_overflowed", (self._spawn_overflow > 0).any(dim=1))

    def __getitem__(self, key):
        if key == "spawn_overflowed":
            self._derive()
        return super().__getitem__(key)

    def __contains__(self, key) -> bool:
        return key == "spawn_overflowed" or super().__contains__(key)

    def get(self, key, default=None):
        return self[key] if key in self else default

    def keys(self):
        self._derive()
        return super().keys()

    def items(self):
        self._derive()
        return super().items()

    def __iter__(self):
        self._derive()
        return super().__iter__()


@dataclasses.dataclass
class SymbolicObservation:
    feature_maps: torch.Tensor  # uint8 [L, H, W, 6]
    scalars: torch.Tensor       # int32 [L, 4]


@dataclasses.dataclass
class EnvironmentState:
    """lifecycle.EnvironmentState (adapters/lifecycle.py:24-31) over L lanes."""

    core_state: State
    environment_root: torch.Tensor  # uint32 [L, 2]
    episode_index: torch.Tensor     # uint32 [L]
    _buffers: dict[str, torch.Tensor] = dataclasses.field(default_factory=dict, repr=False)
    _masks_current: bool = dataclasses.field(default=False, repr=False)
    _launches: int = dataclasses.field(default=0, repr=False)  # alternates the kernel's traversal order
    _cache: dict = dataclasses.field(default_factory=dict, repr=False)  # per-state call structures and views

    @property
    def lanes(self) -> int:
        return int(self.episode_index.shape[0])


@dataclasses.dataclass(frozen=True)
class JaxMARLLayout:
    """adapters/jaxmarl/layout.py:34-67."""

    height: int
    width: int
    per_player_capacity: int
    surface: str
    partial_observability: bool
    final_observation: bool
    action_widths: tuple[int, ...]
    mask_offsets: tuple[int, ...]
    mask_width: int
    feature_maps_dtype: torch.dtype
    mask_form: str = "rows"

    @property
    def agents(self) -> tuple[str, ...]:
        return AGENTS

    @property
    def action_factors(self) -> tuple[str, ...]:
        return ACTION_FACTORS

    @property
    def actions_shape(self) -> tuple[int, int]:
        return (self.per_player_capacity, len(ACTION_FACTORS))

    @property
    def mask_shape(self) -> tuple[int, int]:
        """layout.py:64-67: rows, or the three factor-aligned words of the packed form."""
        return (self.per_player_capacity, self.mask_width if self.mask_form == "rows" else MASK_WORDS)


def make(env_id: str, *, scenario: GameConfig, utt: UnitTypeTableVersion | None = None, surface: str = "symbolic",
         partial_observability: bool = False, final_observation: bool = True, feature_dtype: Any = None,
         reward_components: bool = False, device: Any = None, mask_form: str = "rows") -> NanoRTS:
    """``nanorts.make`` (adapters/jaxmarl/facade.py:43-56).  ``mask_form`` is
    ``jaxmarl.prepare``'s (adapters/jaxmarl/layout.py:70-95): ``"packed"`` makes
    ``get_avail_actions`` return uint32 [L, C, 3] words (adapters/factors.py:89-103)."""
    if env_id not in ENVIRONMENT_IDS:
        raise ModelError(f"make refuses environment id {env_id!r}: the accepted ids are {list(ENVIRONMENT_IDS)}")
    game = scenario if utt is None else _content.with_unit_type_table(scenario, utt)
    return NanoRTS(game, surface=surface, partial_observability=partial_observability,
                   final_observation=final_observation, feature_dtype=feature_dtype,
                   reward_components=reward_components, device=device, mask_form=mask_form)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    assert t.is_contiguous()
    return t.data_ptr()


class NanoRTS:
    """The two-player environment over batches of games on one CUDA device."""

    def __init__(self, scenario: GameConfig, *, surface: str = "symbolic", partial_observability: bool = False,
                 final_observation: bool = True, feature_dtype: Any = None, reward_components: bool = False,
                 device: Any = None, mask_form: str = "rows") -> None:
        if surface != "symbolic":
            raise ModelError(f"NanoRTS refuses surface={surface!r}: this build publishes the symbolic surface only")
        if not isinstance(partial_observability, bool) or not isinstance(final_observation, bool):
            raise ModelError("partial_observability and final_observation must be bools")
        if not isinstance(reward_components, bool):
            raise ModelError(f"NanoRTS refuses reward_components={reward_components!r}: it must be a bool")
        if reward_components and scenario.bucket.unit_type_capacity < 7:
            raise ModelError("reward_components needs the seven standard unit types (adapters/rewards.py:8-27)")
        if feature_dtype is None:
            feature_dtype = torch.uint8
        if feature_dtype not in (torch.uint8, torch.int16, torch.int32):
            raise ModelError(f"feature_dtype {feature_dtype!r} is none of uint8, int16, int32")
        bucket = scenario.bucket
        if mask_form not in MASK_FORMS:
            raise ModelError(f"NanoRTS refuses mask_form={mask_form!r}: a mask publishes one of {list(MASK_FORMS)}")
        if mask_form == "packed" and (ACTION_KIND_COUNT + 4 * DIRECTION_COUNT + bucket.unit_type_capacity > 32
                                      or bucket.attack_offset_capacity > 64):
            raise ModelError("mask_form='packed' needs 6+16+T <= 32 and an attack window of at most 64 cells "
                             "(adapters/factors.py:63-86)")
        if bucket.index_dtype != np.int16:
            raise ModelError("this build steps scenarios whose cell and slot indices fit int16")
        if bucket.width > 64 or bucket.height > 64:
            raise ModelError(f"this build steps fields up to 64x64, not {bucket.height}x{bucket.width}")
        reset = _content.decide(scenario.initial_state, bucket)
        if bool(reset["game_over"]):
            raise ModelError("NanoRTS refuses a scenario whose initial State is already decided")
        self.game = scenario
        self.agents = list(AGENTS)
        self.num_agents = PLAYER_COUNT
        self.final_observation = final_observation
        self.reward_components = reward_components
        self.partial_observability = partial_observability
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        widths = (ACTION_KIND_COUNT, DIRECTION_COUNT, DIRECTION_COUNT, DIRECTION_COUNT, DIRECTION_COUNT,
                  bucket.unit_type_capacity, bucket.attack_offset_capacity)
        offsets = tuple(int(v) for v in np.cumsum((0, *widths[:-1])))
        self.layout = JaxMARLLayout(
            height=bucket.height, width=bucket.width, per_player_capacity=bucket.per_player_capacity,
            surface=surface, partial_observability=partial_observability, final_observation=final_observation,
            action_widths=widths, mask_offsets=offsets, mask_width=sum(widths), feature_maps_dtype=feature_dtype,
            mask_form=mask_form,
        )
        self.packed = mask_form == "packed"
        self._shapes = leaf_shapes(bucket)
        self._extents = Extents(
            height=bucket.height, width=bucket.width, neutral=bucket.neutral_capacity,
            capacity=bucket.per_player_capacity, types=bucket.unit_type_capacity,
            offsets=bucket.attack_offset_capacity, strategy=STRATEGY_CODES[bucket.conflict_strategy],
            max_cycles=scenario.max_cycles, partial_observability=int(partial_observability),
        )
        self._reset_rows = {
            name: torch.from_numpy(np.ascontiguousarray(reset[name]).astype(self._shapes[name][1])).to(self.device)
            for name in LEAVES
        }
        self._content = Content()
        terrain = np.ascontiguousarray(scenario.terrain.reshape(-1).astype(np.uint8))
        table = np.ascontiguousarray(scenario.table, dtype=np.int32)
        check(library().nrts_prepare_scenario(ctypes.byref(self._extents), terrain.ctypes.data, table.ctypes.data,
                                              ctypes.byref(self._content.scenario)))
        for k, name in enumerate(LEAVES):
            self._content.reset[k] = _ptr(self._reset_rows[name])

    # -- buffers ----------------------------------------------------------------
    def _empty_state(self, lanes: int) -> EnvironmentState:
        leaves = {}
        for name in LEAVES:
            shape, dtype, _ = self._shapes[name]
            leaves[name] = torch.empty((lanes, *shape), dtype=_TORCH_DTYPES[np.dtype(dtype)], device=self.device)
        return EnvironmentState(
            core_state=State(**leaves),
            environment_root=torch.empty((lanes, 2), dtype=torch.uint32, device=self.device),
            episode_index=torch.empty((lanes,), dtype=torch.uint32, device=self.device),
        )

    def _buffers(self, state: EnvironmentState) -> dict[str, torch.Tensor]:
        if state._buffers:
            return state._buffers
        L, b, dev = state.lanes, self.game.bucket, self.device
        u8 = torch.uint8
        mask_buffer = (("packed_masks", torch.empty((PLAYER_COUNT, L, b.per_player_capacity, MASK_WORDS), dtype=torch.uint32,
                                                    device=dev)) if self.packed else
                       ("masks", torch.empty((PLAYER_COUNT, L, b.per_player_capacity, self.layout.mask_width), dtype=u8,
                                             device=dev)))
        buf = {
            mask_buffer[0]: mask_buffer[1],
            "feature_maps": torch.empty((PLAYER_COUNT, L, b.height, b.width, 6), dtype=u8, device=dev),
            "scalars": torch.empty((PLAYER_COUNT, L, 4), dtype=torch.int32, device=dev),
            "reward": torch.empty((L, PLAYER_COUNT), dtype=torch.float32, device=dev),
            "done": torch.empty((L,), dtype=u8, device=dev),
            "terminated": torch.empty((L,), dtype=u8, device=dev),
            "truncated": torch.empty((L,), dtype=u8, device=dev),
            "winner": torch.empty((L,), dtype=torch.int32, device=dev),
            "spawn_overflow": torch.empty((L, PLAYER_COUNT), dtype=torch.int32, device=dev),
        }
        if self.final_observation:
            buf["final_feature_maps"] = torch.empty_like(buf["feature_maps"])
            buf["final_scalars"] = torch.empty_like(buf["scalars"])
        if self.reward_components:
            buf["reward_components"] = torch.empty((L, PLAYER_COUNT, 6), dtype=torch.float32, device=dev)
        state._buffers = buf
        return buf

    def _action_buffer(self, state: EnvironmentState, avoid: int | None = None) -> torch.Tensor:
        buf = self._buffers(state)
        for name in ("actions", "actions_alt"):
            if name not in buf:
                buf[name] = torch.empty((PLAYER_COUNT, state.lanes, self.game.bucket.per_player_capacity, 7),
                                        dtype=torch.int32, device=self.device)
        first, second = buf["actions"], buf["actions_alt"]
        in_first = avoid is not None and first.data_ptr() <= avoid < first.data_ptr() + first.numel() * 4
        return second if in_first else first

    def _state_ptrs(self, state: EnvironmentState) -> StatePtrs:
        leaves = state.core_state.leaves()
        key = tuple(leaf.data_ptr() for leaf in leaves) + (state.environment_root.data_ptr(), state.episode_index.data_ptr())
        cached = state._cache.get("ptrs")
        if cached is not None and cached[0] == key:
            return cached[1]
        ptrs = StatePtrs(environment_root=_ptr(state.environment_root), episode_index=_ptr(state.episode_index))
        for k, leaf in enumerate(leaves):
            if leaf.device != self.device or not leaf.is_contiguous():
                raise ModelError("every state leaf must be a contiguous tensor on the environment's device")
            ptrs.leaf[k] = leaf.data_ptr()
        state._cache["ptrs"] = (key, ptrs)
        return ptrs

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _observations(self, buf: dict[str, torch.Tensor], prefix: str = "") -> dict[str, SymbolicObservation]:
        maps, scalars = buf[prefix + "feature_maps"], buf[prefix + "scalars"]
        dtype = self.layout.feature_maps_dtype
        return {
            agent: SymbolicObservation(
                feature_maps=maps[p] if dtype == torch.uint8 else maps[p].to(dtype),
                scalars=scalars[p],
            )
            for p, agent in enumerate(self.agents)
        }

    # -- the JaxMARL surface ----------------------------------------------------
    def reset(self, key: torch.Tensor) -> tuple[dict[str, SymbolicObservation], EnvironmentState]:
        """env.reset over lanes: ``key`` is uint32[L, 2] threefry key data (facade.py:100-105)."""
        key = torch.as_tensor(key)
        if key.ndim != 2 or key.shape[1] != 2:
            raise ModelError(f"reset keys have shape {tuple(key.shape)}, expected [L, 2] key data")
        key = key.to(device=self.device, dtype=torch.uint32).contiguous()
        state = self._empty_state(int(key.shape[0]))
        buf = self._buffers(state)
        out = Outputs()
        self._set_masks(out, buf)
        out.feature_maps[0], out.feature_maps[1] = _ptr(buf["feature_maps"][0]), _ptr(buf["feature_maps"][1])
        out.scalars[0], out.scalars[1] = _ptr(buf["scalars"][0]), _ptr(buf["scalars"][1])
        ptrs = self._state_ptrs(state)
        check(library().nrts_reset(ctypes.byref(self._extents), ctypes.byref(self._content), ctypes.byref(ptrs),
                                   state.lanes, _ptr(key), ctypes.byref(out), self._stream()))
        state._masks_current = True
        return self._observations(buf), state

    def step(self, key: Any, state: EnvironmentState, actions: dict[str, torch.Tensor], reset_state: Any = None, *,
             sample: tuple[int, int] | None = None) -> tuple[dict[str, SymbolicObservation], EnvironmentState, dict, dict, dict]:
        """env.step (facade.py:107-119): the key is ignored, as in the reference.

        ``sample=(seed, counter)`` also draws the next actions inside the same
        kernel from the legality rows it writes (``infos["sampled_actions"]``),
        the values ``sample_actions`` would return for that seed and counter.
        """
        del key
        if reset_state is not None:
            raise ModelError("NanoRTS.step refuses a reset_state: auto-reset restarts each game at its own root")
        buf = self._buffers(state)
        L, C = state.lanes, self.game.bucket.per_player_capacity
        rows = []
        for agent in self.agents:
            a = actions[agent]
            if a.shape != (L, C, 7) or a.dtype != torch.int32 or a.device != self.device or not a.is_contiguous():
                raise ModelError(f"actions[{agent!r}] must be a contiguous int32 tensor [L, {C}, 7] on {self.device}")
            rows.append(a)
        call = state._cache.get("step")
        if call is None:
            call = self._step_call(state, buf)
            state._cache["step"] = call
        out, results = call["outputs"], call["results"]
        infos = results[3]
        if sample is not None:
            # Two action buffers alternate so the draw never overwrites the rows this step reads.
            sampled = self._action_buffer(state, avoid=rows[0].data_ptr())
            out.sampled_actions[0], out.sampled_actions[1] = _ptr(sampled[0]), _ptr(sampled[1])
            out.sample_seed, out.sample_counter = sample[0] & (2**64 - 1), sample[1] & (2**64 - 1)
            infos["sampled_actions"] = {agent: sampled[p] for p, agent in enumerate(self.agents)}
        else:
            out.sampled_actions[0] = out.sampled_actions[1] = None
            infos.pop("sampled_actions", None)
        out.reverse_order = state._launches & 1
        state._launches += 1
        infos.stale()
        ptrs = self._state_ptrs(state)
        check(library().nrts_step(ctypes.byref(self._extents), ctypes.byref(self._content), ctypes.byref(ptrs), L,
                                  _ptr(rows[0]), _ptr(rows[1]), ctypes.byref(out), self._stream()))
        state._masks_current = True
        observations, rewards, dones = results[0], results[1], results[2]
        if self.layout.feature_maps_dtype != torch.uint8:  # converted copies, not views: fresh every step
            observations = self._observations(buf)
            if self.final_observation:
                infos["final_observation"] = self._observations(buf, "final_")
        return observations, state, rewards, dones, infos

    def _step_call(self, state: EnvironmentState, buf: dict[str, torch.Tensor]) -> dict:
        """The Outputs struct and the returned views of one state's buffers, built once."""
        out = Outputs()
        self._set_masks(out, buf)
        for p in range(PLAYER_COUNT):
            out.feature_maps[p] = _ptr(buf["feature_maps"][p])
            out.scalars[p] = _ptr(buf["scalars"][p])
            if self.final_observation:
                out.final_feature_maps[p] = _ptr(buf["final_feature_maps"][p])
                out.final_scalars[p] = _ptr(buf["final_scalars"][p])
        for name in ("reward", "done", "terminated", "truncated", "winner", "spawn_overflow"):
            setattr(out, name, _ptr(buf[name]))
        if self.reward_components:
            out.reward_components = _ptr(buf["reward_components"])
        done = buf["done"].view(torch.bool)
        rewards = {agent: buf["reward"][:, p] for p, agent in enumerate(self.agents)}
        dones = {agent: done for agent in self.agents} | {ALL_AGENTS: done}
        infos = StepInfos(buf["spawn_overflow"])
        infos.update({
            "terminated": buf["terminated"].view(torch.bool),
            "truncated": buf["truncated"].view(torch.bool),
            "winner": buf["winner"],
            "telemetry": Telemetry(spawn_overflow=buf["spawn_overflow"]),
            "final_valid": done,
        })
        if self.final_observation:
            infos["final_observation"] = self._observations(buf, "final_")
        if self.reward_components:  # facade.py:220-223, adapters/rewards.py:20-27 order
            infos["reward_components"] = {agent: buf["reward_components"][:, p] for p, agent in enumerate(self.agents)}
        return {"outputs": out, "results": (self._observations(buf), rewards, dones, infos)}

    def _set_masks(self, out: Outputs, buf: dict[str, torch.Tensor]) -> None:
        name = "packed_masks" if self.packed else "masks"
        target = out.packed_masks if self.packed else out.masks
        target[0], target[1] = _ptr(buf[name][0]), _ptr(buf[name][1])

    def get_avail_actions(self, state: EnvironmentState) -> dict[str, torch.Tensor]:
        """bool[L, C, 78] per agent (facade.py:172-174), or uint32[L, C, 3] words with
        mask_form="packed"; reuses what the last step wrote."""
        buf = self._buffers(state)
        if self.packed:
            if not state._masks_current:
                ptrs = self._state_ptrs(state)
                check(library().nrts_packed_masks(ctypes.byref(self._extents), ctypes.byref(self._content),
                                                  ctypes.byref(ptrs), state.lanes, _ptr(buf["packed_masks"][0]),
                                                  _ptr(buf["packed_masks"][1]), self._stream()))
                state._masks_current = True
            return {agent: buf["packed_masks"][p] for p, agent in enumerate(self.agents)}
        if not state._masks_current:
            ptrs = self._state_ptrs(state)
            check(library().nrts_legal_masks(ctypes.byref(self._extents), ctypes.byref(self._content),
                                             ctypes.byref(ptrs), state.lanes, _ptr(buf["masks"][0]),
                                             _ptr(buf["masks"][1]), self._stream()))
            state._masks_current = True
        return {agent: buf["masks"][p].view(torch.bool) for p, agent in enumerate(self.agents)}

    def _row_masks(self, state: EnvironmentState) -> dict[str, torch.Tensor]:
        """Byte rows of the current state whatever the mask form (the standalone sampler reads rows)."""
        if not self.packed:
            return self.get_avail_actions(state)
        buf = self._buffers(state)
        if "masks" not in buf:
            buf["masks"] = torch.empty((PLAYER_COUNT, state.lanes, self.game.bucket.per_player_capacity,
                                        self.layout.mask_width), dtype=torch.uint8, device=self.device)
        ptrs = self._state_ptrs(state)
        check(library().nrts_legal_masks(ctypes.byref(self._extents), ctypes.byref(self._content), ctypes.byref(ptrs),
                                         state.lanes, _ptr(buf["masks"][0]), _ptr(buf["masks"][1]), self._stream()))
        return {agent: buf["masks"][p].view(torch.bool) for p, agent in enumerate(self.agents)}

    def check_device(self) -> None:
        """Waits for this environment's stream and raises DeviceStatusError when
        a kernel on the device recorded that a bounded staging wait gave up
        (the status word is read and cleared; it is shared by every call on
        the device)."""
        torch.cuda.current_stream(self.device).synchronize()
        check_device(self.device.index if self.device.index is not None else torch.cuda.current_device())

    def invalidate(self, state: EnvironmentState) -> None:
        """Marks cached masks stale after the caller edited the state's leaves."""
        state._masks_current = False

    def get_obs(self, state: EnvironmentState) -> dict[str, SymbolicObservation]:
        """facade.py:166-170."""
        buf = self._buffers(state)
        ptrs = self._state_ptrs(state)
        check(library().nrts_observe(ctypes.byref(self._extents), ctypes.byref(self._content), ctypes.byref(ptrs),
                                     state.lanes, _ptr(buf["feature_maps"][0]), _ptr(buf["feature_maps"][1]),
                                     _ptr(buf["scalars"][0]), _ptr(buf["scalars"][1]), self._stream()))
        return self._observations(buf)

    def get_slot_cells(self, state: EnvironmentState) -> dict[str, torch.Tensor]:
        """int32[L, C] per agent, -1 for an empty slot (facade.py:176-178)."""
        L, C = state.lanes, self.game.bucket.per_player_capacity
        cells = torch.empty((L, PLAYER_COUNT, C), dtype=torch.int32, device=self.device)
        ptrs = self._state_ptrs(state)
        check(library().nrts_slot_cells(ctypes.byref(self._extents), ctypes.byref(ptrs), L, _ptr(cells), self._stream()))
        return {agent: cells[:, p] for p, agent in enumerate(self.agents)}

    def sample_actions(self, state: EnvironmentState, seed: int, counter: int) -> dict[str, torch.Tensor]:
        """Uniform legal actions per factor from the current masks (the rollout stand-in for
        per-factor categorical sampling over masked logits, README.md:53-63)."""
        masks = self._row_masks(state)
        acts = self._action_buffer(state)
        check(library().nrts_sample_actions(ctypes.byref(self._extents), state.lanes, _ptr(masks["player_0"]),
                                            _ptr(masks["player_1"]), _ptr(acts[0]), _ptr(acts[1]),
                                            seed & (2**64 - 1), counter & (2**64 - 1), self._stream()))
        return {agent: acts[p] for p, agent in enumerate(self.agents)}

    def observation_space(self, agent: str) -> dict[str, Any]:
        return {"feature_maps": ((self.layout.height, self.layout.width, 6), self.layout.feature_maps_dtype),
                "scalars": ((4,), torch.int32)}

    def action_space(self, agent: str) -> dict[str, Any]:
        return {"shape": self.layout.actions_shape, "high": tuple(w - 1 for w in self.layout.action_widths)}

    @property
    def agent_classes(self) -> dict[str, list[str]]:
        return {"player": list(self.agents)}

    def idle_row(self) -> torch.Tensor:
        row = torch.zeros(self.layout.mask_width, dtype=torch.bool)
        row[self.layout.mask_offsets[0] + KIND_NONE] = True
        return row


def unpack_mask(words: torch.Tensor, layout: JaxMARLLayout) -> torch.Tensor:
    """adapters/factors.py:106-114 unpack: packed uint32 [..., 3] words -> bool [..., 78] rows."""
    if layout.mask_form != "packed":
        return words
    head = sum(layout.action_widths[:-1])
    shifts = torch.arange(32, device=words.device, dtype=torch.int64)
    bits = ((words.to(torch.int64)[..., None] >> shifts) & 1).bool().reshape(*words.shape[:-1], MASK_WORDS * 32)
    return torch.cat([bits[..., :head], bits[..., 32:32 + layout.action_widths[-1]]], dim=-1)
