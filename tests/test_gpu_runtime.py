"""Device self check and the bounded-wait status path (needs a B200).

The staging waits of every kernel are bounded: after the limit a wait records
the device status word and returns, leaving the context usable.  The self
check exercises that path on an mbarrier nothing ever completes (1 ms limit),
with no fault, trap or hang; the host then reads the status through
nrts_device_status.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.parity import CONFIGS, random_keys

pytestmark = pytest.mark.gpu


def test_self_check_gives_up_a_bounded_wait_and_keeps_the_status():
    from nanorts_b200.runtime import check, library

    lib = library()
    assert lib.nrts_device_status(0) == 0  # nothing failed before (and the word is cleared)
    devices = (ctypes.c_int32 * 1)(0)
    check(lib.nrts_self_check(devices, 1))
    # The probe's timeout was recorded and then the earlier value (0) restored.
    assert lib.nrts_device_status(0) == 0


def test_steps_run_after_the_self_check():
    """The context stays usable after a wait gave up: a reset and steps run and
    leave no status behind."""
    from nanorts_b200.env import make
    from nanorts_b200.runtime import check, library

    lib = library()
    check(lib.nrts_self_check((ctypes.c_int32 * 1)(0), 1))
    game = CONFIGS["c2_16x16_random"].game(50)
    env = make("NanoRTS", scenario=game, final_observation=False)
    keys = random_keys(np.random.default_rng(2), 64)
    _, state = env.reset(torch.from_numpy(keys.view(np.int32)).cuda().view(torch.uint32))
    for t in range(5):
        env.step(None, state, env.sample_actions(state, seed=0, counter=t))
    torch.cuda.synchronize()
    assert lib.nrts_device_status(0) == 0
