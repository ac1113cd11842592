"""TEST INFRASTRUCTURE ONLY: where the reference (packed-encoders 0.3.0) source tree is, and its
Python package installed into ``baseline/_ref`` for the tests and the bench's reference arm.

The tree is taken from the ``PE_REFERENCE_DIR`` environment variable, else from a ``reference``
checkout beside this repository. ``pip install --target baseline/_ref`` of the reference fails
offline (its build backend, hatchling, is not available), so ``install_reference_package``
copies the files its wheel would hold (``[tool.hatch.build.targets.wheel] packages =
["packed_encoders"]`` in its pyproject.toml): the pure-Python package plus the C sources its CPU
loader compiles at run time. ``baseline/_ref`` is git-ignored and travels to the GPU box with the
repository snapshot; nothing on the GPU box reads the reference tree itself.
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
BASELINE = ROOT / "baseline" / "_ref"


def reference_dir() -> Path | None:
    """The reference source tree (the directory that holds ``packed_encoders/``), or None."""
    env = os.environ.get("PE_REFERENCE_DIR")
    candidates = [Path(env)] if env else []
    candidates.append(ROOT.parent / "reference")
    for cand in candidates:
        if (cand / "packed_encoders" / "__init__.py").exists():
            return cand.resolve()
    return None


def install_reference_package(dest: Path = BASELINE) -> Path | None:
    """Copy the reference package into ``dest`` (replacing an older copy); None without a tree."""
    src = reference_dir()
    if src is None:
        return None
    target = dest / "packed_encoders"
    staging = dest / "packed_encoders.tmp"
    if staging.exists():
        shutil.rmtree(staging)
    dest.mkdir(parents=True, exist_ok=True)
    shutil.copytree(src / "packed_encoders", staging, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    if target.exists():
        shutil.rmtree(target)
    staging.rename(target)
    (dest / "SOURCE.txt").write_text(f"copied from {src} (packed-encoders package tree, pip build unavailable)\n")
    return target


def add_reference_to_path() -> bool:
    """Put the installed reference package on ``sys.path``; True when ``baseline/_ref`` holds it."""
    if not (BASELINE / "packed_encoders" / "__init__.py").exists():
        return False
    if str(BASELINE) not in sys.path:
        sys.path.append(str(BASELINE))
    return True
