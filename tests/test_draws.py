"""The oracle's threefry composition, pinned to published and reference vectors.

* threefry2x32 (20 rounds) against the Random123 known-answer vectors (the
  values JAX's own test suite checks its threefry_2x32 against);
* fold_in / the conflict draw against golden vectors generated from the
  reference's own core/cuda/conflict_draw.cuh (tests/golden/make_draws.py);
* against that reference build directly when it was built here.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import pytest

GOLDEN = json.loads((Path(__file__).parent / "golden" / "conflict_draws.json").read_text())

KAT = [
    ((0x00000000, 0x00000000), (0x00000000, 0x00000000), (0x6B200159, 0x99BA4EFE)),
    ((0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF), (0x1CB996FC, 0xBB002BE7)),
    ((0x13198A2E, 0x03707344), (0x243F6A88, 0x85A308D3), (0xC4923A9C, 0x483DF7A0)),
]


def _threefry(lib, k, x):
    a, b = ctypes.c_uint32(x[0]), ctypes.c_uint32(x[1])
    lib.oracle_threefry2x32(k[0], k[1], ctypes.addressof(a), ctypes.addressof(b))
    return a.value, b.value


@pytest.mark.parametrize("key,counter,expected", KAT)
def test_threefry_known_answers(oracle_lib, key, counter, expected):
    assert _threefry(oracle_lib.lib(), key, counter) == expected


def test_threefry_golden_blocks(oracle_lib):
    lib = oracle_lib.lib()
    for k0, k1, x0, x1, y0, y1 in GOLDEN["threefry2x32"]:
        assert _threefry(lib, (k0, k1), (x0, x1)) == (y0, y1)


def test_fold_in_golden(oracle_lib):
    lib = oracle_lib.lib()
    for k0, k1, data, y0, y1 in GOLDEN["fold_in"]:
        out = (ctypes.c_uint32 * 2)()
        lib.oracle_fold_in(k0, k1, data, out)
        assert (out[0], out[1]) == (y0, y1)


def test_conflict_draws_golden(oracle_lib):
    lib = oracle_lib.lib()
    values = set()
    for k0, k1, time, birth, ordinal, draw in GOLDEN["conflict_draws"]:
        assert lib.oracle_conflict_draw(k0, k1, time, birth, ordinal) == draw
        values.add(draw)
    assert values == {0, 1}


def test_against_reference_build(oracle_lib):
    ref = oracle_lib.ref_draws()
    if ref is None:
        pytest.skip("the reference's conflict_draw.cuh was not built here (oracle/_ref)")
    lib = oracle_lib.lib()
    for k0 in range(0, 2**32, 2**28 + 12345):
        for time in (0, 1, 777, 4999):
            for birth in (0, 5, 131):
                for ordinal in range(4):
                    assert lib.oracle_conflict_draw(k0, k0 ^ 0x5A5A, time, birth, ordinal) == \
                        ref.ref_conflict_draw(k0, k0 ^ 0x5A5A, time, birth, ordinal)
