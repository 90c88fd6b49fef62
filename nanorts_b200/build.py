"""Builds the in-tree sm_100a library with nvcc.

``python -m nanorts_b200.build`` or ``nanorts_b200.build.build()`` compiles
``csrc/*.cu`` into ``_lib/libnanorts_b200.so`` (cross-compiles without a GPU).
The build is skipped when the library is newer than every source.
``build_ffi()`` adds ``_lib/libnanorts_b200_ffi.so``, the jax.ffi handlers,
where jaxlib's XLA FFI header is available.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCES = sorted((HERE / "csrc").glob("*.cu"))
HEADERS = sorted((HERE / "csrc").glob("*.cuh")) + [HERE.parent / "include" / "nanorts_b200.h"]
OUTPUT = HERE / "_lib" / "libnanorts_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not OUTPUT.exists():
        return True
    built = OUTPUT.stat().st_mtime
    return any(path.stat().st_mtime > built for path in (*SOURCES, *HEADERS, Path(__file__)))


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    command = [_nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", str(tmp), *map(str, SOURCES)]
    subprocess.run(command, check=True)
    tmp.replace(OUTPUT)
    return OUTPUT


FFI_SOURCE = HERE / "ffi" / "nanorts_b200_ffi.cc"
FFI_OUTPUT = HERE / "_lib" / "libnanorts_b200_ffi.so"


def xla_ffi_include() -> Path | None:
    """The directory holding jaxlib's ``xla/ffi/api/ffi.h``: ``XLA_FFI_INCLUDE``
    when set, else ``jax.ffi.include_dir()`` when jax is importable, else None."""
    named = os.environ.get("XLA_FFI_INCLUDE")
    candidates = [Path(named)] if named else []
    if not named:
        try:
            import jax.ffi  # noqa: PLC0415 - optional

            candidates.append(Path(jax.ffi.include_dir()))
        except Exception:  # noqa: BLE001 - jax absent or without ffi
            pass
    for root in candidates:
        if (root / "xla" / "ffi" / "api" / "ffi.h").is_file():
            return root
    return None


def build_ffi(force: bool = False, include: Path | None = None) -> Path | None:
    """Compiles the jax.ffi handlers (ffi/nanorts_b200_ffi.cc) into
    ``_lib/libnanorts_b200_ffi.so``, linked with the step library, where
    jaxlib's XLA FFI header is found; returns None (and builds nothing) where
    it is not."""
    include = include or xla_ffi_include()
    if include is None:
        return None
    library = build()
    if not force and FFI_OUTPUT.exists() and FFI_OUTPUT.stat().st_mtime > max(
            FFI_SOURCE.stat().st_mtime, library.stat().st_mtime, Path(__file__).stat().st_mtime):
        return FFI_OUTPUT
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    cuda_include = Path(_nvcc()).resolve().parent.parent / "include"
    tmp = FFI_OUTPUT.with_suffix(".so.tmp")
    command = [cxx, "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{include}", f"-I{HERE.parent / 'include'}",
               f"-I{cuda_include}", "-o", str(tmp), str(FFI_SOURCE), f"-L{library.parent}", "-lnanorts_b200",
               "-Wl,-rpath,$ORIGIN"]
    subprocess.run(command, check=True)
    tmp.replace(FFI_OUTPUT)
    return FFI_OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_ffi(force="--force" in sys.argv) or "jax.ffi handlers skipped: no xla/ffi/api/ffi.h (jaxlib) found")
