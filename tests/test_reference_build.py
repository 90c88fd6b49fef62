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


def test_reference_path_stand_ins_match_the_oracle():
    """The torch stand-ins for the reference's XLA fusions that drive its
    kernels in the timing path (decode_actions, the uniform draw) agree with
    the oracle on random-play states of configs 1, 2 and 5."""
    import numpy as np
    import torch

    from oracle import ref_kernels as rk
    from oracle.oracle import Oracle
    from tests.parity import CONFIGS, random_keys, sample

    for name, lanes in (("c2_16x16_random", 12), ("c1_8x8_both", 12), ("c5_64x64_random", 3)):
        game = CONFIGS[name].game(200)
        orc = Oracle(game, lanes)
        rng = np.random.default_rng(1)
        orc.reset(random_keys(rng, lanes))
        widths = (6, 4, 4, 4, 4, game.bucket.unit_type_capacity, game.bucket.attack_offset_capacity)
        for t in range(40):
            masks = orc.legal_masks()
            actions = sample(masks, rng, 0.4)
            leaves = {n: torch.from_numpy(orc.state[n].copy()) for n in rk.LEAVES}
            got = torch.stack(rk.decode_actions(leaves, torch.from_numpy(actions), game.bucket), 1).numpy()
            assert np.array_equal(got, orc.decode_actions(actions)), f"{name} step {t}: decode"
            drawn = rk.sample_uniform(torch.from_numpy(masks.astype(bool)), widths).numpy()
            start = 0
            for f, w in enumerate(widths):
                group = masks[..., start:start + w]
                picked = np.take_along_axis(group, drawn[..., f:f + 1].astype(np.int64), -1)[..., 0]
                assert np.all(~group.any(-1) | (picked == 1)), f"{name} step {t}: factor {f} drew an illegal value"
                start += w
            orc.step(actions)
