"""Loads the sm_100a library and binds its C ABI (include/nanorts_b200.h).

The library is built in-tree (``nanorts_b200/_lib/libnanorts_b200.so``) by
``nanorts_b200.build``.  There is no fallback: when the library is missing or
fails to load, every entry point raises ``KernelUnavailable``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "_lib" / "libnanorts_b200.so"

LEAF_COUNT = 23


class KernelUnavailable(RuntimeError):
    """The CUDA library is not built or cannot load; no CPU path exists."""


class KernelError(RuntimeError):
    """A C-ABI call returned an error code."""


class Extents(ctypes.Structure):
    _fields_ = [
        ("height", ctypes.c_int32), ("width", ctypes.c_int32), ("neutral", ctypes.c_int32),
        ("capacity", ctypes.c_int32), ("types", ctypes.c_int32), ("offsets", ctypes.c_int32),
        ("strategy", ctypes.c_int32), ("max_cycles", ctypes.c_int32), ("partial_observability", ctypes.c_int32),
    ]


MAX_HEIGHT, MAX_TYPES, TABLE_COLUMNS = 64, 8, 15


class Scenario(ctypes.Structure):
    _fields_ = [
        ("terrain_rows", ctypes.c_uint64 * MAX_HEIGHT), ("attack_window", ctypes.c_uint64 * MAX_TYPES),
        ("producible", ctypes.c_uint32 * MAX_TYPES), ("resource_types", ctypes.c_uint32),
        ("stockpile_types", ctypes.c_uint32), ("table", ctypes.c_int32 * (MAX_TYPES * (TABLE_COLUMNS + MAX_TYPES))),
    ]


class Content(ctypes.Structure):
    _fields_ = [("scenario", Scenario), ("reset", ctypes.c_void_p * LEAF_COUNT)]


class StatePtrs(ctypes.Structure):
    _fields_ = [("leaf", ctypes.c_void_p * LEAF_COUNT), ("environment_root", ctypes.c_void_p),
                ("episode_index", ctypes.c_void_p)]


class Outputs(ctypes.Structure):
    _fields_ = [
        ("masks", ctypes.c_void_p * 2), ("feature_maps", ctypes.c_void_p * 2), ("scalars", ctypes.c_void_p * 2),
        ("reward", ctypes.c_void_p), ("done", ctypes.c_void_p), ("terminated", ctypes.c_void_p),
        ("truncated", ctypes.c_void_p), ("winner", ctypes.c_void_p), ("spawn_overflow", ctypes.c_void_p),
        ("final_feature_maps", ctypes.c_void_p * 2), ("final_scalars", ctypes.c_void_p * 2),
        ("sampled_actions", ctypes.c_void_p * 2), ("sample_seed", ctypes.c_uint64), ("sample_counter", ctypes.c_uint64),
        ("reward_components", ctypes.c_void_p), ("packed_masks", ctypes.c_void_p * 2), ("reverse_order", ctypes.c_uint32),
    ]


class GroupStep(ctypes.Structure):
    """NrtsGroupStep: one group of a multi-group step."""
    _fields_ = [("extents", ctypes.c_void_p), ("content", ctypes.c_void_p), ("state", ctypes.c_void_p),
                ("lanes", ctypes.c_int64), ("actions", ctypes.c_void_p * 2), ("outputs", ctypes.c_void_p)]


MAX_GROUPS = 8
CARRY_FIELDS = 9


class BotCarry(ctypes.Structure):
    _fields_ = [("field", ctypes.c_void_p * CARRY_FIELDS), ("trained", ctypes.c_void_p), ("next_order", ctypes.c_void_p)]


class BotSpec(ctypes.Structure):
    """NrtsBot: strategy, trained unit type, carry."""
    _fields_ = [("strategy", ctypes.c_int32), ("trained", ctypes.c_int32), ("carry", BotCarry)]


# Every symbol the header declares.
SYMBOLS = (
    "nrts_prepare_scenario", "nrts_step", "nrts_step_groups", "nrts_reset", "nrts_legal_masks", "nrts_packed_masks", "nrts_observe",
    "nrts_slot_cells", "nrts_sample_actions",
    "nrts_bot_act", "nrts_duel_step", "nrts_device_status", "nrts_build_id", "nrts_self_check", "nrts_self_check_no_alloc",
    "nrts_last_error",
)

_LIB: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """The loaded library; raises KernelUnavailable when it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY.exists():
        raise KernelUnavailable(f"{LIBRARY} is not built; run nanorts_b200.build.build()")
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError as error:
        raise KernelUnavailable(f"cannot load {LIBRARY}: {error}") from error
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.nrts_prepare_scenario.argtypes = [p, p, p, p]
    lib.nrts_step.argtypes = [p, p, p, i64, p, p, p, p]
    lib.nrts_reset.argtypes = [p, p, p, i64, p, p, p]
    lib.nrts_step_groups.argtypes = [p, i32, p]
    lib.nrts_legal_masks.argtypes = [p, p, p, i64, p, p, p]
    lib.nrts_packed_masks.argtypes = [p, p, p, i64, p, p, p]
    lib.nrts_observe.argtypes = [p, p, p, i64, p, p, p, p, p]
    lib.nrts_slot_cells.argtypes = [p, p, i64, p, p]
    lib.nrts_sample_actions.argtypes = [p, i64, p, p, p, p, ctypes.c_uint64, ctypes.c_uint64, p]
    lib.nrts_bot_act.argtypes = [p, p, p, i64, i32, p, p, p]
    lib.nrts_duel_step.argtypes = [p, p, p, i64, p, p, p]
    lib.nrts_device_status.argtypes = [ctypes.c_int]
    lib.nrts_self_check.argtypes = [p, i64]
    lib.nrts_self_check_no_alloc.argtypes = [p, i64]
    lib.nrts_build_id.restype = ctypes.c_char_p
    lib.nrts_last_error.restype = ctypes.c_char_p
    for name in ("nrts_prepare_scenario", "nrts_step", "nrts_step_groups", "nrts_reset", "nrts_legal_masks", "nrts_packed_masks", "nrts_observe",
                 "nrts_slot_cells",
                 "nrts_sample_actions", "nrts_bot_act", "nrts_duel_step", "nrts_device_status", "nrts_self_check",
                 "nrts_self_check_no_alloc"):
        getattr(lib, name).restype = i32
    _LIB = lib
    return lib


class DeviceStatusError(KernelError):
    """A kernel's bounded wait gave up: the games it had not stepped are stale."""


def check_device(device_index: int) -> None:
    """Reads and clears the device status word (nrts_device_status, synchronous);
    raises DeviceStatusError when a kernel recorded that a bounded wait gave up."""
    status = check(library().nrts_device_status(device_index))
    if status != 0:
        raise DeviceStatusError(f"device {device_index}: a kernel's bounded wait gave up (status {status}); "
                                "the games of that launch's remaining warps were not stepped")


def check(code: int) -> int:
    if code < 0:
        message = library().nrts_last_error().decode()
        raise KernelError(f"nanorts_b200 call failed ({code}): {message}")
    return code
