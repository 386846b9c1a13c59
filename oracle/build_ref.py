"""Puts the reference's own Python package where the CPU baseline can import it (test infrastructure).

The reference (`qwen38_inf2`) is pure Python with no packaging files, so "building" it is a copy of its
package directory, unmodified, into oracle/_ref/ (git-ignored, carried to the GPU box with the rest of
the working tree). bench.py's reference arm then times the reference's own CPU branches from there.
Nothing in the product imports it. Run from a checkout that has the reference:

    python oracle/build_ref.py [--reference /path/to/reference]
"""

from __future__ import annotations

import argparse
import shutil
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def build(reference: str | Path | None = None) -> Path | None:
    """Copies <reference>/qwen38_inf2 to oracle/_ref/qwen38_inf2; returns the target, or None when the
    reference checkout is not present (the GPU box keeps the copy made before it was sent there)."""
    src = Path(reference) / "qwen38_inf2" if reference else None
    if src is None or not src.is_dir():
        return TARGET if (TARGET / "qwen38_inf2").is_dir() else None
    dst = TARGET / "qwen38_inf2"
    if dst.exists():
        shutil.rmtree(dst)
    TARGET.mkdir(exist_ok=True)
    shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    return TARGET


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    print(build(ap.parse_args().reference))
