"""Install infrared (xiangzhang-coding/infrared, the reference) for the checks
that run its own code — TEST INFRASTRUCTURE ONLY.

infrared is pure Python on PyTorch. Its checkout is installed, unmodified,
with pip (no index, no build isolation, no dependencies: torch is already
present) into ``baseline/_ref`` of this repository. That directory is
git-ignored, so none of the reference's source enters the history, but it
travels with the repository to a GPU box, where

* the ``-m gpu`` engine tests run infrared's ``PagedBatchEngine`` (eager and
  CUDA-graph decode, chunked prefill, preemption) with the shim installed
  and compare its greedy tokens with infrared's own paths;
* ``bench.py --impl reference`` and the ``cpu_baseline`` leg time infrared's
  own naive attention (``paged_attention(..., use_triton=False)``) on the
  host cores;
* ``bench.py --config c5 --engine`` decodes through infrared's engine.

The product (``infrared_b200``) never imports infrared; the shim only patches
it when a caller installs it.

Usage: ``python -m oracle.reference_install [SRC]`` where ``SRC`` (or the
``INFRARED_SRC`` environment variable) is an infrared checkout; the pip
build writes into its source tree, so it runs on a temporary copy.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
TARGET = ROOT / "baseline" / "_ref"


def installed(target: Path = TARGET) -> bool:
    return (target / "infrared" / "__init__.py").exists()


def default_source() -> Path | None:
    """``INFRARED_SRC``, else a checkout named ``reference`` beside this
    repository (the layout of the build machine); None if neither exists."""
    env = os.environ.get("INFRARED_SRC")
    cands = [Path(env)] if env else [ROOT.parent / "reference"]
    for c in cands:
        if (c / "infrared" / "__init__.py").exists() and (c / "pyproject.toml").exists():
            return c
    return None


def install(src: Path | None = None, target: Path = TARGET, force: bool = False) -> bool:
    """pip-install the checkout ``src`` into ``target``; False if there is no
    checkout to install from (nothing changes then)."""
    if installed(target) and not force:
        return True
    src = Path(src) if src is not None else default_source()
    if src is None:
        return False
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "infrared-src"
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        if target.exists():
            shutil.rmtree(target)
        target.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index",
                        "--no-build-isolation", "--no-deps", "--quiet", "--target", str(target),
                        str(copy)], check=True)
    return installed(target)


if __name__ == "__main__":
    ok = install(Path(sys.argv[1]) if len(sys.argv) > 1 else None, force="--force" in sys.argv)
    print(TARGET if ok else "no infrared checkout found (pass SRC or set INFRARED_SRC)")
