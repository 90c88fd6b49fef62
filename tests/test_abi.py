"""The C ABI without a GPU: the library loads, exports every symbol
include/nanorts_b200.h declares, prepares scenarios on the host and refuses
bad arguments before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from nanorts_b200 import map_name_to_scenario, runtime
from nanorts_b200.model import STRATEGY_CODES

HEADER = Path(__file__).resolve().parents[1] / "include" / "nanorts_b200.h"


@pytest.fixture(scope="module")
def lib():
    from nanorts_b200 import build

    build.build()
    return runtime.library()


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nrts_[a-z_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert "nrts_step" in names and "nrts_prepare_scenario" in names
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(runtime.SYMBOLS) == names


def test_ctypes_layouts_match_the_header(lib, tmp_path):
    """Struct sizes and offsets as a C compiler lays the header out."""
    import shutil
    import subprocess

    compiler = shutil.which("gcc") or shutil.which("cc")
    if compiler is None:
        pytest.skip("no C compiler")
    probe = tmp_path / "layout.c"
    probe.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "nanorts_b200.h"\n'
        "int main(void) { printf(\"%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(NrtsExtents), "
        "sizeof(NrtsScenario), sizeof(NrtsContent), sizeof(NrtsState), sizeof(NrtsOutputs), "
        "offsetof(NrtsOutputs, sampled_actions), offsetof(NrtsScenario, table), sizeof(NrtsBotCarry), "
        "sizeof(NrtsBot), offsetof(NrtsBot, carry)); return 0; }\n")
    exe = tmp_path / "layout"
    subprocess.run([compiler, "-I", str(HEADER.parent), str(probe), "-o", str(exe)], check=True)
    sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert sizes == [ctypes.sizeof(runtime.Extents), ctypes.sizeof(runtime.Scenario), ctypes.sizeof(runtime.Content),
                     ctypes.sizeof(runtime.StatePtrs), ctypes.sizeof(runtime.Outputs),
                     runtime.Outputs.sampled_actions.offset, runtime.Scenario.table.offset,
                     ctypes.sizeof(runtime.BotCarry), ctypes.sizeof(runtime.BotSpec), runtime.BotSpec.carry.offset]


def extents_of(game) -> runtime.Extents:
    b = game.bucket
    return runtime.Extents(height=b.height, width=b.width, neutral=b.neutral_capacity, capacity=b.per_player_capacity,
                           types=b.unit_type_capacity, offsets=b.attack_offset_capacity,
                           strategy=STRATEGY_CODES[b.conflict_strategy], max_cycles=game.max_cycles)


def test_prepare_scenario_packs_terrain_and_tables(lib):
    game = map_name_to_scenario("GardenOfWar64x64", capacity_profile=False, utt="VERSION_ORIGINAL")
    x = extents_of(game)
    sc = runtime.Scenario()
    terrain = np.ascontiguousarray(game.terrain.reshape(-1).astype(np.uint8))
    table = np.ascontiguousarray(game.table)
    assert lib.nrts_prepare_scenario(ctypes.byref(x), terrain.ctypes.data, table.ctypes.data, ctypes.byref(sc)) == 0
    for y in range(64):
        row = int(sc.terrain_rows[y])
        assert [(row >> xx) & 1 for xx in range(64)] == list(game.terrain[y].astype(int))
    assert sc.producible[1] == 1 << 3  # Base -> Worker
    assert sc.producible[3] == (1 << 1) | (1 << 2)  # Worker -> Base, Barracks
    assert sc.resource_types == 1 and sc.stockpile_types == 1 << 1
    assert bin(sc.attack_window[6]).count("1") == 29  # Ranged: range 3 disk in the 7x7 window
    assert bin(sc.attack_window[3]).count("1") == 5  # Worker: range 1
    assert sc.attack_window[1] == 0  # a Base cannot attack


@pytest.mark.parametrize("field,value", [("width", 65), ("types", 9), ("offsets", 48), ("strategy", 3), ("capacity", 0)])
def test_bad_extents_are_refused(lib, field, value):
    game = map_name_to_scenario("basesWorkers8x8")
    x = extents_of(game)
    setattr(x, field, value)
    sc = runtime.Scenario()
    terrain = np.zeros(64, np.uint8)
    rc = lib.nrts_prepare_scenario(ctypes.byref(x), terrain.ctypes.data, game.table.ctypes.data, ctypes.byref(sc))
    assert rc == -1
    assert lib.nrts_last_error().decode()


def test_null_state_is_refused_before_any_launch(lib):
    game = map_name_to_scenario("basesWorkers8x8")
    x = extents_of(game)
    content = runtime.Content()
    assert lib.nrts_step(ctypes.byref(x), ctypes.byref(content), None, 4, None, None, None, None) == -1
    assert "null" in lib.nrts_last_error().decode()


def _dummy_state_and_content(game):
    """Host buffers standing in for device pointers: every call below is refused before any launch."""
    keep = [np.zeros(4096, np.int32) for _ in range(2 * runtime.LEAF_COUNT + 2)]
    state, content = runtime.StatePtrs(), runtime.Content()
    for k in range(runtime.LEAF_COUNT):
        state.leaf[k] = keep[k].ctypes.data
        content.reset[k] = keep[runtime.LEAF_COUNT + k].ctypes.data
    state.environment_root, state.episode_index = keep[-2].ctypes.data, keep[-1].ctypes.data
    return state, content, keep


@pytest.mark.parametrize("strategy,trained,message", [(2, -1, "strategy"), (1, 7, "trained"), (1, -1, "trained")])
def test_bad_bots_are_refused_before_any_launch(lib, strategy, trained, message):
    game = map_name_to_scenario("basesWorkers8x8")
    x = extents_of(game)
    state, content, keep = _dummy_state_and_content(game)
    bot = runtime.BotSpec(strategy=strategy, trained=trained)
    for f in range(runtime.CARRY_FIELDS):
        bot.carry.field[f] = keep[0].ctypes.data
    bot.carry.trained = bot.carry.next_order = keep[0].ctypes.data
    bots = (runtime.BotSpec * 2)(bot, bot)
    out = runtime.Outputs()
    assert lib.nrts_duel_step(ctypes.byref(x), ctypes.byref(content), ctypes.byref(state), 4, bots, ctypes.byref(out), None) == -1
    assert message in lib.nrts_last_error().decode()
    assert lib.nrts_bot_act(ctypes.byref(x), ctypes.byref(content), ctypes.byref(state), 4, 0, ctypes.byref(bot),
                            keep[0].ctypes.data, None) == -1
    assert lib.nrts_bot_act(ctypes.byref(x), ctypes.byref(content), ctypes.byref(state), 4, 2, ctypes.byref(bot),
                            keep[0].ctypes.data, None) == -1
    assert "player" in lib.nrts_last_error().decode()


def test_null_carry_is_refused(lib):
    game = map_name_to_scenario("basesWorkers8x8")
    x = extents_of(game)
    state, content, keep = _dummy_state_and_content(game)
    bot = runtime.BotSpec(strategy=0, trained=-1)
    out = runtime.Outputs()
    bots = (runtime.BotSpec * 2)(bot, bot)
    assert lib.nrts_duel_step(ctypes.byref(x), ctypes.byref(content), ctypes.byref(state), 4, bots, ctypes.byref(out), None) == -1
    assert "carry" in lib.nrts_last_error().decode()


def test_negative_lane_counts_are_refused(lib):
    """nrts_sample_actions and nrts_slot_cells refuse lanes < 0 as every other
    entry point does, before any launch."""
    game = map_name_to_scenario("basesWorkers8x8")
    x = extents_of(game)
    state, content, keep = _dummy_state_and_content(game)
    buf = keep[0].ctypes.data
    assert lib.nrts_sample_actions(ctypes.byref(x), -1, buf, buf, buf, buf, 0, 0, None) == -1
    assert "negative" in lib.nrts_last_error().decode()
    assert lib.nrts_slot_cells(ctypes.byref(x), ctypes.byref(state), -3, buf, None) == -1
    assert "negative" in lib.nrts_last_error().decode()
    out = runtime.Outputs()
    assert lib.nrts_step(ctypes.byref(x), ctypes.byref(content), ctypes.byref(state), -2, buf, buf, ctypes.byref(out),
                         None) == -1
    assert "negative" in lib.nrts_last_error().decode()


def test_no_alloc_self_check_refuses_device_lists_beyond_its_limits(lib):
    """More than 64 devices, a negative count or an index outside 0..63 is
    refused before any device work."""
    devices = (ctypes.c_int32 * 65)(*([0] * 65))
    assert lib.nrts_self_check_no_alloc(devices, 65) == -1
    assert "64 devices" in lib.nrts_last_error().decode()
    assert lib.nrts_self_check_no_alloc(devices, -1) == -1
    assert lib.nrts_self_check_no_alloc(None, 1) == -1
    assert "null" in lib.nrts_last_error().decode()
    assert lib.nrts_self_check_no_alloc((ctypes.c_int32 * 1)(64), 1) == -1
    assert "0..63" in lib.nrts_last_error().decode()


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(runtime, "LIBRARY", tmp_path / "absent.so")
    monkeypatch.setattr(runtime, "_LIB", None)
    with pytest.raises(runtime.KernelUnavailable):
        runtime.library()

