"""jax.ffi custom calls over the sm_100a kernels (needs jax with jaxlib's XLA FFI).

``register()`` loads ``_lib/libnanorts_b200_ffi.so`` (built by
``nanorts_b200.build.build_ffi()`` where jaxlib's ``xla/ffi/api/ffi.h`` is
found) and registers its handlers as CUDA FFI targets, as NanoRTS registers
its own library (``src/nanorts/kernels/library.py:27-69``).  ``scenario_attributes``
and ``reset_operands`` give what every call passes besides the State: the
scenario as attributes and one game's reset State as shared-row operands
(no device pointer lives in an attribute, so a traced executable runs on any
device).  Operand and result orders are documented in
``ffi/nanorts_b200_ffi.cc``.

JAX is not part of this image, so the binding is exercised in the tests by
driving the same handlers through an XLA FFI interface stand-in
(``tests/test_gpu_jax_ffi.py``).
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from nanorts_b200 import content as _content
from nanorts_b200.model import STRATEGY_CODES, GameConfig, leaf_shapes

TARGETS = ("nanorts_b200_step", "nanorts_b200_reset", "nanorts_b200_legal_masks", "nanorts_b200_observe",
           "nanorts_b200_bot_act")

LEAVES = (
    "birth", "unit_type", "owner", "cell", "hit_points", "carried_resources", "pending_kind", "pending_direction",
    "pending_none_duration", "pending_target_cell", "pending_produced_type", "pending_issued_at",
    "pending_completes_at", "pending_order", "entity_at", "time", "player_resources", "next_birth",
    "next_pending_order", "alternating_conflict_count", "game_over", "winner", "spawn_overflow",
)


class JaxUnavailable(RuntimeError):
    """jax (with jaxlib's XLA FFI) or the handler library is not available."""


_HANDLE: ctypes.CDLL | None = None


def register() -> ctypes.CDLL:
    """Builds (where possible) and registers the handlers as jax.ffi CUDA targets."""
    global _HANDLE
    if _HANDLE is not None:
        return _HANDLE
    try:
        import jax
    except ImportError as error:
        raise JaxUnavailable("jax is not installed; the jax.ffi binding needs jax and jaxlib") from error
    from nanorts_b200 import build

    library = build.build_ffi()
    if library is None:
        raise JaxUnavailable("jaxlib's xla/ffi/api/ffi.h was not found; set XLA_FFI_INCLUDE")
    handle = ctypes.CDLL(str(library))
    for name in TARGETS:
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(handle, name)), platform="CUDA")
    _HANDLE = handle
    return handle


def scenario_attributes(game: GameConfig, partial_observability: bool = False) -> dict[str, Any]:
    """The attributes every handler takes (int64 extents, int32 terrain and unit table)."""
    b = game.bucket
    return {
        "height": np.int64(b.height), "width": np.int64(b.width), "neutral": np.int64(b.neutral_capacity),
        "capacity": np.int64(b.per_player_capacity), "types": np.int64(b.unit_type_capacity),
        "offsets": np.int64(b.attack_offset_capacity), "strategy": np.int64(STRATEGY_CODES[b.conflict_strategy]),
        "max_cycles": np.int64(game.max_cycles), "partial_observability": np.int64(int(partial_observability)),
        "terrain": np.ascontiguousarray(game.terrain.reshape(-1), dtype=np.int32),
        "table": np.ascontiguousarray(game.table.reshape(-1), dtype=np.int32),
    }


def reset_operands(game: GameConfig) -> list[np.ndarray]:
    """One game's reset State (decide(initial_state)) as shared rows [1, ...], in leaf order."""
    reset = _content.decide(game.initial_state, game.bucket)
    shapes = leaf_shapes(game.bucket)
    return [np.ascontiguousarray(reset[name], dtype=shapes[name][1]).reshape(1, *shapes[name][0]) for name in LEAVES]


def step(state_leaves, environment_root, episode_index, actions0, actions1, game: GameConfig,
         partial_observability: bool = False):
    """``nanorts_b200_step`` as one ``jax.ffi.ffi_call`` (state aliased in
    place, as the reference's own step target aliases it, core/cycle.py:131)."""
    import jax
    import jax.numpy as jnp

    register()
    b = game.bucket
    L, C, H, W = state_leaves[0].shape[0], b.per_player_capacity, b.height, b.width
    state = [*state_leaves, environment_root, episode_index]
    results = [jax.ShapeDtypeStruct(x.shape, x.dtype) for x in state]
    results += [jax.ShapeDtypeStruct((L, C, b.mask_width), jnp.bool_)] * 2
    results += [jax.ShapeDtypeStruct((L, H, W, 6), jnp.uint8)] * 2
    results += [jax.ShapeDtypeStruct((L, 4), jnp.int32)] * 2
    results += [jax.ShapeDtypeStruct((L, 2), jnp.float32), *[jax.ShapeDtypeStruct((L,), jnp.bool_)] * 3,
                jax.ShapeDtypeStruct((L,), jnp.int32), jax.ShapeDtypeStruct((L, 2), jnp.int32)]
    call = jax.ffi.ffi_call("nanorts_b200_step", results, input_output_aliases={k: k for k in range(len(state))})
    return call(*state, *[jnp.asarray(r) for r in reset_operands(game)], actions0, actions1,
                **scenario_attributes(game, partial_observability))
