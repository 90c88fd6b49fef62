"""nrts_self_check_no_alloc against nrts_self_check (needs a B200).

Some callers of this library cannot allocate device memory: in a JAX process
XLA's client takes most or all of each GPU's memory for its own allocator at
start-up, so a cudaMalloc made behind its back can fail, and a custom call is
meant to draw memory only from XLA.  nrts_self_check allocates a small buffer
for its probe results; nrts_self_check_no_alloc writes them into a static
device array of the library instead.  Both must give the same answer, call
after call, since the array keeps the previous call's contents.

This file is collected last (its name sorts after every other test file), so
a run that stops at the first failure has run every other test before it.  It
passes alone in a fresh process, where its first call also does the one-time
set-up for device 0, and after the other tests.
"""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


def test_no_alloc_self_check_agrees_with_the_allocating_one_on_two_calls():
    from nanorts_b200.runtime import library

    lib = library()
    devices = (ctypes.c_int32 * 1)(0)
    expected = lib.nrts_self_check(devices, 1)
    assert expected == 0, lib.nrts_last_error()
    for call in range(2):
        got = lib.nrts_self_check_no_alloc(devices, 1)
        assert got == expected, f"call {call}: {lib.nrts_last_error()}"
    # The probes' bounded wait records into the static array, not into the
    # library's status word.
    assert lib.nrts_device_status(0) == 0
