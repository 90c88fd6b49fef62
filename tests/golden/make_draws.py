"""Generates tests/golden/conflict_draws.json from the reference's own
conflict-draw composition (core/cuda/conflict_draw.cuh of NanoRTS, built as
host code into oracle/_ref/libref_draws.so by `make -C oracle ref`).

Each record: root key (k0, k1), time, birth, ordinal, the fold_in chain's
event key and the draw.  Run from the repository root:
    python tests/golden/make_draws.py
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]


def main() -> None:
    ref = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_draws.so"))
    ref.ref_conflict_draw.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
    ref.ref_conflict_draw.restype = ctypes.c_int32
    ref.ref_fold_in.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, ctypes.c_void_p]
    ref.ref_threefry2x32.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
    rng = np.random.default_rng(20261201)
    draws, folds, blocks = [], [], []
    for _ in range(256):
        k0, k1 = (int(v) for v in rng.integers(0, 2**32, 2, dtype=np.uint64))
        time, birth, ordinal = int(rng.integers(0, 5000)), int(rng.integers(0, 3000)), int(rng.integers(0, 8))
        draws.append([k0, k1, time, birth, ordinal, int(ref.ref_conflict_draw(k0, k1, time, birth, ordinal))])
    for _ in range(64):
        k0, k1, data = (int(v) for v in rng.integers(0, 2**31, 3, dtype=np.uint64))
        out = (ctypes.c_uint32 * 2)()
        ref.ref_fold_in(k0, k1, data, out)
        folds.append([k0, k1, data, int(out[0]), int(out[1])])
    for _ in range(64):
        k0, k1, x0, x1 = (int(v) for v in rng.integers(0, 2**32, 4, dtype=np.uint64))
        a, b = ctypes.c_uint32(x0), ctypes.c_uint32(x1)
        ref.ref_threefry2x32(k0, k1, ctypes.byref(a), ctypes.byref(b))
        blocks.append([k0, k1, x0, x1, a.value, b.value])
    out = {"source": "reference core/cuda/conflict_draw.cuh (host build)", "conflict_draws": draws, "fold_in": folds,
           "threefry2x32": blocks}
    (ROOT / "tests" / "golden" / "conflict_draws.json").write_text(json.dumps(out))
    print(f"wrote {len(draws)} draws, {len(folds)} fold_ins, {len(blocks)} blocks")


if __name__ == "__main__":
    main()
