"""Slab layouts of the launches, checked on the host (no GPU).

The kernels stage a game's State rows and their scratch in one shared-memory
slab whose offsets `make_layout` (csrc/step.cu) computes.  TMA bulk copies
need 16-byte-aligned destinations, the mbarrier an 8-byte-aligned word, and
regions that alias one another in time must each fit before the mbarrier.  A
host-only probe (tests/layout_probe.cu, built once into tests/_build/) prints
the layouts each launch shape uses for the benchmark maps, and these tests
check those rules and the games per SM the launch shapes rely on.
"""

from __future__ import annotations

import json
import shutil
import subprocess
from pathlib import Path

import pytest

from nanorts_b200 import map_name_to_scenario

ROOT = Path(__file__).resolve().parents[1]
PROBE_SRC = ROOT / "tests" / "layout_probe.cu"
PROBE = ROOT / "tests" / "_build" / "layout_probe"
SOURCES = [PROBE_SRC, *sorted((ROOT / "nanorts_b200" / "csrc").glob("*")), ROOT / "include" / "nanorts_b200.h"]

SMEM_PER_BLOCK = 232_448   # opt-in dynamic shared memory per CTA on sm_100
SMEM_PER_SM = 233_472      # shared memory per SM
CTA_RESERVE = 1_024        # shared memory the runtime reserves per CTA


@pytest.fixture(scope="module")
def probe() -> Path:
    nvcc = shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not found")
    if not PROBE.exists() or PROBE.stat().st_mtime < max(p.stat().st_mtime for p in SOURCES):
        PROBE.parent.mkdir(parents=True, exist_ok=True)
        # PTX only: the probe runs no kernel, it only needs the host code.
        subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=compute_100a", "-I", str(ROOT / "include"),
                        "-o", str(PROBE), str(PROBE_SRC)], check=True, capture_output=True)
    return PROBE


def extents(map_name: str, **kw):
    b = map_name_to_scenario(map_name, **kw).bucket
    return (b.height, b.width, b.neutral_capacity, b.per_player_capacity, b.unit_type_capacity, b.attack_offset_capacity)


def layout(probe: Path, ext, aligned: bool, bots: bool, hbm: bool, compact: bool) -> dict:
    args = [str(v) for v in ext] + [str(int(aligned)), str(int(bots)), str(int(hbm)), str(int(compact))]
    return json.loads(subprocess.run([str(probe), *args], check=True, capture_output=True, text=True).stdout)


# (map, scenario keywords, row alignment of the benchmark's batches)
MAPS = {
    "8x8": ("basesWorkers8x8", {}, True),
    "16x16": ("basesWorkers16x16", {}, True),
    "64x64": ("GardenOfWar64x64", {"capacity_profile": False}, False),
    "15wide": ("itsNotSafe", {"capacity_profile": False}, False),
}
# Launch shapes: the step kernels, the compact wide-board kernel (rules-only
# rows in HBM), the bot kernels (rules-only rows in HBM, bot scratch).
SHAPES = {"step": (False, False, False), "wide_compact": (False, True, True), "bots": (True, True, False)}


@pytest.mark.parametrize("shape", sorted(SHAPES))
@pytest.mark.parametrize("board", sorted(MAPS))
def test_layout_rules(probe, board, shape):
    name, kw, aligned = MAPS[board]
    ext = extents(name, **kw)
    H, W, N, C = ext[:4]
    E, owned, cells = N + 2 * C, 2 * C, H * W
    bots, hbm, compact = SHAPES[shape]
    L = layout(probe, ext, aligned, bots, hbm, compact)
    bar, slab = L["bar_off"], L["slab_bytes"]
    assert slab % 16 == 0 and bar % 8 == 0 and bar + 16 <= slab
    assert L["header_bytes"] + slab <= SMEM_PER_BLOCK
    # Staged rows: 16-byte-aligned slots in leaf order, room for the unaligned
    # head and tail when rows are not 16-byte multiples, all below the scalars.
    end = 0
    for off, size in zip(L["leaf_off"], L["row_bytes"]):
        if off < 0:
            continue
        assert off % 16 == 0 and off >= end
        end = off + size + (0 if aligned else 16)
    assert end <= L["scal_off"]
    names = ["scal_off", "list_off", "order_off", "scan_off", "conf_off", "key_off", "info_off", "rank_off", "count_off",
             "free_off", "member_key_off", "ret_off", "word_off", "rows_off", "mask_off"]
    if bots:
        names += ["carry_off", "cmd_off", "bot_off"]
    for n in names:
        assert L[n] % 16 == 0, n
    # Admission: the contested ranks (int16 [2C]) lie over the claim counts,
    # whose region must hold them; everything ends before the mbarrier.
    count_bytes = L["claim_words"] * 4 + 8 + 2 * 5 * 4
    assert L["serial_off"] == L["count_off"]
    assert L["count_off"] + max(count_bytes, 2 * owned) <= bar
    assert L["scan_off"] + 2 * E <= L["conf_off"] and L["conf_off"] + 2 * E <= L["key_off"]
    assert L["info_off"] + 12 * owned <= L["rank_off"] and L["rank_off"] + 2 * owned <= L["count_off"]
    # Completion and the epilogue, aliasing the admission scratch.
    assert L["ret_off"] + 20 * owned <= bar
    assert L["rows_off"] - L["word_off"] >= 4 * (E if compact else cells)
    assert L["mask_off"] - L["rows_off"] >= 4 * H * 8
    assert L["mask_off"] + 4 * (3 * owned + 6) <= bar
    if bots:
        assert L["bot_off"] + L["bot_bytes"] <= bar
        assert L["carry_off"] < L["cmd_off"] <= L["bot_off"]


def test_games_per_sm_of_the_benchmark_launches(probe):
    """The residency the launch shapes are sized for: up to 24 games per SM
    for 16x16 steps (one CTA per SM), five 64x64 games per SM in the compact
    layout (one CTA each), twenty 16x16 bot games per SM."""
    step16 = layout(probe, extents("basesWorkers16x16"), True, False, False, False)
    assert (SMEM_PER_BLOCK - step16["header_bytes"]) // step16["slab_bytes"] >= 24
    wide = layout(probe, extents("GardenOfWar64x64", capacity_profile=False), False, False, True, True)
    assert 5 * (wide["slab_bytes"] + wide["header_bytes"] + CTA_RESERVE) <= SMEM_PER_SM
    duel = layout(probe, extents("basesWorkers16x16"), True, True, True, False)
    assert (SMEM_PER_BLOCK - duel["header_bytes"]) // duel["slab_bytes"] >= 20
