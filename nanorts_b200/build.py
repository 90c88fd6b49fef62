"""Builds the in-tree sm_100a library with nvcc.

``python -m nanorts_b200.build`` or ``nanorts_b200.build.build()`` compiles
``csrc/*.cu`` into ``_lib/libnanorts_b200.so`` (cross-compiles without a GPU).
The build is skipped when the library is newer than every source.
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


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
