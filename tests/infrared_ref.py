"""Where the tests find infrared (xiangzhang-coding/infrared), the reference.

``INFRARED_REF`` names a directory that holds the ``infrared`` package (a
checkout, or a pip ``--target`` install); by default the repository's own
git-ignored install ``baseline/_ref`` (made by ``oracle/reference_install.py``,
which ``__graft_entry__.build()`` runs), which travels to a GPU box with the
repository. Tests that need infrared skip when neither is present.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def location() -> str | None:
    env = os.environ.get("INFRARED_REF")
    cand = Path(env) if env else ROOT / "baseline" / "_ref"
    return str(cand) if (cand / "infrared" / "__init__.py").exists() else None


def importable() -> bool:
    path = location()
    if path is None:
        return False
    if path not in sys.path:
        sys.path.insert(0, path)
    return True
