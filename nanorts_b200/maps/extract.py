"""Convert NanoRTS's shipped MicroRTS map XMLs into ``maps.json``.

Usage: ``python -m nanorts_b200.maps.extract <nanorts source tree>/src/nanorts/maps``

Every map up to 64x64 is kept (the kernels address rows as 64-bit words).
Each record holds the parsed document: width, height, terrain digits, the
two player records and the units in document order, which is the order the
loader claims slots and assigns births in.
"""

from __future__ import annotations

import dataclasses
import json
import sys
from pathlib import Path

from nanorts_b200.content import document_from_xml

MAX_EXTENT = 64


def main(root: str) -> None:
    maps = {}
    for path in sorted(Path(root).rglob("*.xml")):
        document = document_from_xml(path.read_text(encoding="utf-8"))
        if document.width > MAX_EXTENT or document.height > MAX_EXTENT:
            continue
        maps[path.stem] = {
            "width": document.width,
            "height": document.height,
            "terrain": document.terrain,
            "players": [list(p) for p in document.players],
            "units": [list(dataclasses.astuple(u)) for u in document.units],
        }
    out = Path(__file__).resolve().parent / "maps.json"
    out.write_text(json.dumps(maps, separators=(",", ":"), sort_keys=True))
    print(f"wrote {len(maps)} maps to {out}")


if __name__ == "__main__":
    main(sys.argv[1])
