"""
Recipe: the reference's own Python code as a CPU baseline that travels.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

    python oracle/ref_build.py <reference checkout>

The reference is pure Python (no build step of its own). This recipe copies
its two packages, unmodified, into ``oracle/_ref/``: ``create_graph`` (from
``src/create_graph``) and ``kernels`` (``kernels/edge_attn``, its example op).
``oracle/_ref/`` is git-ignored, so the reference's sources never enter this
repository's history, but it travels with the working tree to the GPU box,
where bench.py's CPU-baseline and reference legs import the reference's own
``cg.create_graph`` and ``EdgeAttention`` from it (oracle/ref.py). Without it
those legs time the oracle's restatement instead and say so.
"""

from __future__ import annotations

import pathlib
import shutil
import sys

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"


def build(reference_root: str | pathlib.Path) -> bool:
    """Copy the reference packages into oracle/_ref; False when the checkout is absent."""
    root = pathlib.Path(reference_root)
    src, kernels = root / "src" / "create_graph", root / "kernels"
    if not (src / "__init__.py").exists() or not (kernels / "edge_attn" / "ops.py").exists():
        return False
    OUT.mkdir(exist_ok=True)
    for from_dir, name in ((src, "create_graph"), (kernels, "kernels")):
        dest = OUT / name
        if dest.exists():
            shutil.rmtree(dest)
        shutil.copytree(from_dir, dest, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    for extra in ("LICENSE",):
        if (root / extra).exists():
            shutil.copy2(root / extra, OUT / extra)
    return True


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    print("copied" if build(sys.argv[1]) else "reference checkout not found", OUT)
