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
