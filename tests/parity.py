"""Shared helpers of the parity tests: the kernel path and the CPU oracle
stepped side by side on identical seeded action streams."""

from __future__ import annotations

import dataclasses

import numpy as np

from nanorts_b200 import content
from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion

WIDTHS = (6, 4, 4, 4, 4, 7, 49)


@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    map: str
    utt: UnitTypeTableVersion
    strategy: ConflictStrategy
    partial: bool = False
    capacity_profile: bool = True
    max_cycles: int = 5000

    def game(self, max_cycles: int | None = None):
        return content.map_name_to_scenario(
            self.map, utt=self.utt, conflict_strategy=self.strategy,
            max_cycles=self.max_cycles if max_cycles is None else max_cycles,
            capacity_profile=self.capacity_profile,
        )


O, F = UnitTypeTableVersion.ORIGINAL, UnitTypeTableVersion.ORIGINAL_FINETUNED
CONFIGS = {
    # The five benchmark configurations' scenarios (configs 1, 2, 3 and 5; config 4 is bot play).
    "c1_8x8_both": Config("c1_8x8_both", "basesWorkers8x8", O, ConflictStrategy.CANCEL_BOTH),
    "c2_16x16_random": Config("c2_16x16_random", "basesWorkers16x16", O, ConflictStrategy.CANCEL_RANDOM),
    "c3_16x16_alternating_partial": Config("c3_16x16_alternating_partial", "basesWorkers16x16", F,
                                           ConflictStrategy.CANCEL_ALTERNATING, partial=True),
    "c5_64x64_random": Config("c5_64x64_random", "GardenOfWar64x64", O, ConflictStrategy.CANCEL_RANDOM,
                              capacity_profile=False),
    # A wide board with partial observability: the visibility rows of the one-game-per-CTA kernel.
    "c5_64x64_alternating_partial": Config("c5_64x64_alternating_partial", "GardenOfWar64x64", F,
                                           ConflictStrategy.CANCEL_ALTERNATING, partial=True, capacity_profile=False),
}


def sample(masks: np.ndarray, rng: np.random.Generator, move_bias: float = 0.0) -> np.ndarray:
    """Uniform legal values per factor; with ``move_bias`` the kind factor picks
    MOVE (or PRODUCE) whenever legal with that probability, which drives units
    into contested cells and exercises the conflict rules."""
    from oracle.oracle import sample_uniform_legal

    actions = sample_uniform_legal(masks, WIDTHS, rng)
    if move_bias > 0:
        claim = np.where(masks[..., 4] != 0, 4, np.where(masks[..., 1] != 0, 1, actions[..., 0]))
        biased = rng.random(actions.shape[:-1]) < move_bias
        actions[..., 0] = np.where(biased, claim, actions[..., 0])
    return actions


def random_keys(rng: np.random.Generator, lanes: int) -> np.ndarray:
    return rng.integers(0, 2**32, size=(lanes, 2), dtype=np.uint64).astype(np.uint32)
