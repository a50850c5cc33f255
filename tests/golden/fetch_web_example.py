"""Copies the reference's example scene (instantsplat-rs/web/example: splat.ply with 222,909
SH-degree-0 Gaussians, cameras.json with 6 cameras of 392 x 518, input_view0..5.png) from a
reference tree into tests/golden/web_example/, where the GPU tests and bench.py read it.

The scene is the reference's own timing scene (instantsplat-rs/examples/step_timing.rs) and
the only one its published step time (instantsplat-rs/src/gpu.rs:22-25) was measured on. At
18 MB it is too large to commit as a fixture: the copy is listed in .gitignore, travels with
the working tree to the GPU machines, and is re-made by __graft_entry__.build() wherever the
reference tree is present. Files are copied byte for byte; nothing is converted.

    python tests/golden/fetch_web_example.py <reference root>
"""

from __future__ import annotations

import hashlib
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "web_example"
FILES = ["splat.ply", "cameras.json"] + [f"input_view{i}.png" for i in range(6)]


def source_of(reference_root: Path) -> Path:
    return Path(reference_root) / "instantsplat-rs" / "web" / "example"


def fetch(reference_root) -> Path | None:
    """Copies the files that are missing or differ; returns the target folder, or None when
    the reference tree does not hold the scene."""
    source = source_of(reference_root)
    if not all((source / name).is_file() for name in FILES):
        return None
    TARGET.mkdir(exist_ok=True)
    for name in FILES:
        src, dst = source / name, TARGET / name
        if dst.is_file() and dst.stat().st_size == src.stat().st_size and _digest(dst) == _digest(src):
            continue
        shutil.copyfile(src, dst)
    return TARGET


def _digest(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def available() -> bool:
    """Whether the copy is complete (the GPU tests and the benchmark skip the scene otherwise)."""
    return all((TARGET / name).is_file() for name in FILES)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    out = fetch(Path(sys.argv[1]))
    print(out if out else "the reference tree holds no web/example scene")
