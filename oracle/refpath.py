"""Where the reference checkout lives, for the checker builds and fixture scripts.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The path comes from the ``QVGGT_REFERENCE`` environment variable, else from the
``reference_path`` field of ``BASELINE.json`` at the repository root (the
benchmark description that names the reference).  Nothing on the product path,
in the GPU tests, ``smoke()`` or ``bench.py`` reads the reference checkout.
"""
from __future__ import annotations

import json
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_path() -> str | None:
    """The reference checkout directory, or None when it is not present."""
    p = os.environ.get("QVGGT_REFERENCE")
    if not p:
        try:
            with open(os.path.join(ROOT, "BASELINE.json")) as f:
                p = json.load(f).get("reference_path")
        except (OSError, ValueError):
            p = None
    return p if p and os.path.isdir(p) else None
