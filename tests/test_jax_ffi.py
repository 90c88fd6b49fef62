"""The jax.ffi handlers (nanorts_b200/ffi/nanorts_b200_ffi.cc) without a GPU.

jaxlib is absent from this image, so the product build of the handlers is
skipped (build_ffi returns None) and register() refuses with a clear error;
the handler source is compiled here against the XLA FFI interface stand-in
(oracle/ffi_standin) with the test harness, which the GPU tests then use to
drive the handlers with real device buffers.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HANDLERS = ("nanorts_b200_step", "nanorts_b200_reset", "nanorts_b200_legal_masks", "nanorts_b200_observe",
            "nanorts_b200_bot_act")


def build_shim(out_dir: Path) -> Path:
    """Handlers + harness against the stand-in, linked with the step library."""
    from nanorts_b200 import build

    library = build.build()
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    cuda_include = Path(build._nvcc()).resolve().parent.parent / "include"
    out = out_dir / "libshim_harness.so"
    subprocess.run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Werror",
                    f"-I{ROOT / 'oracle' / 'ffi_standin'}", f"-I{ROOT / 'include'}", f"-I{cuda_include}", "-o", str(out),
                    str(ROOT / "nanorts_b200" / "ffi" / "nanorts_b200_ffi.cc"),
                    str(ROOT / "tests" / "ffi_harness" / "shim_harness.cc"), f"-L{library.parent}", "-lnanorts_b200",
                    f"-Wl,-rpath,{library.parent}"], check=True)
    return out


def test_product_build_is_skipped_without_jaxlib(tmp_path, monkeypatch):
    from nanorts_b200 import build, jax_binding

    monkeypatch.setenv("XLA_FFI_INCLUDE", str(tmp_path))  # holds no xla/ffi/api/ffi.h
    assert build.xla_ffi_include() is None
    assert build.build_ffi() is None
    monkeypatch.setattr(jax_binding, "_HANDLE", None)
    with pytest.raises(jax_binding.JaxUnavailable):
        jax_binding.register()


def test_handlers_compile_against_the_ffi_interface(tmp_path):
    import ctypes

    lib = ctypes.CDLL(str(build_shim(tmp_path)))
    for name in HANDLERS:
        assert hasattr(lib, f"{name}_implementation"), name
    assert hasattr(lib, "shim_call")


def test_scenario_attributes_and_reset_operands():
    from nanorts_b200 import jax_binding, map_name_to_scenario

    game = map_name_to_scenario("basesWorkers16x16", utt="VERSION_ORIGINAL", conflict_strategy="CANCEL_RANDOM")
    attrs = jax_binding.scenario_attributes(game)
    assert attrs["terrain"].shape == (256,) and attrs["table"].shape == (7 * 22,)
    assert int(attrs["strategy"]) == 1 and int(attrs["capacity"]) == 70
    rows = jax_binding.reset_operands(game)
    assert len(rows) == 23 and all(r.shape[0] == 1 for r in rows)


def test_handlers_refuse_malformed_calls_before_any_launch(tmp_path):
    """The handlers validate operand and result counts, sizes and aliasing on
    the host and return InvalidArgument, as the reference's handlers do
    (core/cuda/step.cu:658-660); nothing reaches the device."""
    import ctypes

    import numpy as np

    from nanorts_b200 import jax_binding, map_name_to_scenario
    from nanorts_b200.model import leaf_shapes

    lib = ctypes.CDLL(str(build_shim(tmp_path)))
    p, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.shim_call.argtypes = [ctypes.c_int32, p, p, i64, p, i64, p, p, i64, p, i64]
    lib.shim_last_error.restype = ctypes.c_char_p

    class Buf(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                    ("dims", ctypes.c_int64 * 6)]

    game = map_name_to_scenario("basesWorkers8x8", utt="VERSION_ORIGINAL")
    attrs = jax_binding.scenario_attributes(game)
    ints = np.array([int(attrs[k]) for k in ("height", "width", "neutral", "capacity", "types", "offsets", "strategy",
                                             "max_cycles", "partial_observability")] + [0, 0, 0], np.int64)
    L = 2
    keep = []

    def buf(shape, itemsize=4, dtype=4):
        a = np.zeros(int(np.prod(shape)) * itemsize, np.uint8)
        keep.append(a)
        b = Buf(data=a.ctypes.data, dtype=dtype, rank=len(shape))
        for k, n in enumerate(shape):
            b.dims[k] = n
        return b

    shapes = leaf_shapes(game.bucket)
    state = [buf((L, *shapes[n][0]), shapes[n][1].itemsize) for n in jax_binding.LEAVES]
    state += [buf((L, 2)), buf((L,))]
    resets = [buf((1, *shapes[n][0]), shapes[n][1].itemsize) for n in jax_binding.LEAVES]

    def call(target, args, rets):
        a, r = (Buf * len(args))(*args), (Buf * max(len(rets), 1))(*rets)
        rc = lib.shim_call(target, None, a, len(args), r, len(rets), ints.ctypes.data, attrs["terrain"].ctypes.data,
                           attrs["terrain"].size, attrs["table"].ctypes.data, attrs["table"].size)
        return rc, lib.shim_last_error().decode()

    rc, msg = call(0, state[:10], [])
    assert rc == 3 and "too few operands" in msg
    rc, msg = call(0, state + resets + [buf((L, 47, 7))] * 2, state)  # too few results
    assert rc == 3 and "50 operands" in msg
    other = [buf((L, *shapes[n][0]), shapes[n][1].itemsize) for n in jax_binding.LEAVES] + [buf((L, 2)), buf((L,))]
    outs = [buf((L, 47, 78), 1)] * 2 + [buf((L, 8, 8, 6), 1)] * 2 + [buf((L, 4))] * 2
    outs += [buf((L, 2)), buf((L,), 1), buf((L,), 1), buf((L,), 1), buf((L,)), buf((L, 2))]
    rc, msg = call(0, state + resets + [buf((L, 47, 7))] * 2, other + outs)
    assert rc == 3 and "alias" in msg
    rc, msg = call(0, state + resets + [buf((L, 46, 7))] * 2, state + outs)
    assert rc == 3 and "actions" in msg
    rc, msg = call(2, state + [buf((2, 1))] + resets[1:], [buf((L, 47, 78), 1)] * 2)
    assert rc == 3 and "shared rows" in msg
