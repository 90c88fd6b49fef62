"""The reference-kernel harness (oracle/ref_kernels.cu): built from the
reference's own sources, it loads and exports every entry point the GPU
reference-parity tests call.  No GPU work is done here."""

from __future__ import annotations

import ctypes

import pytest


def test_reference_kernel_harness_exports_its_entry_points():
    from oracle import ref_kernels

    if not ref_kernels.available():
        pytest.skip("the reference kernels are not built (make -C oracle ref with a NanoRTS checkout)")
    lib = ctypes.CDLL(str(ref_kernels.LIBRARY))
    for name in ("ref_step", "ref_legality_words", "ref_legality_rows", "ref_visible_cells",
                 "ref_reset_packed_where_done", "ref_last_error",
                 # the handlers of the reference sources, exported by the FFI stand-in
                 "nanorts_step_implementation", "nanorts_legality_words_implementation",
                 "nanorts_visible_cells_implementation", "nanorts_reset_packed_where_done_implementation"):
        assert hasattr(lib, name), name


def test_reference_table_columns_follow_unit_tables():
    """The operand tables handed to the reference kernels carry its column
    order (core/unit_tables.py:9-27) for the product's unit table."""
    from nanorts_b200 import map_name_to_scenario
    from oracle import ref_kernels

    game = map_name_to_scenario("basesWorkers16x16")
    ref = ref_kernels.ReferenceKernels(game, device="cpu")
    T = game.bucket.unit_type_capacity
    assert tuple(ref.table.shape) == (1, T, 7 + T) and tuple(ref.timings.shape) == (1, T, 7)
    worker = 3
    assert ref.table[0, worker, :7].tolist() == [1, 1, 0, 0, 1, 1, 1]  # moves, harvests, attacks, range 1, cost 1
    assert ref.timings[0, worker].tolist() == [10, 20, 5, 50, 1, 1, 1]
    assert ref.table[0, 1, 7 + worker] == 1  # a base produces workers
