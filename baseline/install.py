"""Installs the unmodified reference (``wcrmu/MDL``) under ``baseline/_ref`` for the
reference arm of ``bench.py``.

The reference ships neither ``setup.py`` nor ``pyproject.toml``, so pip refuses the
source directory as it is. The install therefore copies the sources to a temporary
directory, adds a minimal ``pyproject.toml`` that only declares the packages ``src`` and
``src.modules``, and runs ``pip install --no-index --no-build-isolation --no-deps
--find-links /opt/wheelhouse --target baseline/_ref`` on that copy. The installed
``src/`` is then compared file by file with the reference sources; any difference
fails the install.

The reference sources are found through ``MDL_REFERENCE_SRC`` or, by default, in the
directory ``reference`` beside this repository's directory.
"""

from __future__ import annotations

import filecmp
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
TARGET = os.path.join(HERE, "_ref")

_PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "mdl-reference"
version = "0.0.0"

[tool.setuptools]
packages = ["src", "src.modules"]
"""


def reference_source() -> str:
    return os.environ.get("MDL_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference"))


def _same_tree(a: str, b: str) -> bool:
    cmp = filecmp.dircmp(a, b, ignore=["__pycache__"])
    if cmp.left_only or cmp.right_only or cmp.funny_files:
        return False
    _match, mismatch, errors = filecmp.cmpfiles(a, b, cmp.common_files, shallow=False)
    if mismatch or errors:
        return False
    return all(_same_tree(os.path.join(a, d), os.path.join(b, d)) for d in cmp.common_dirs)


def installed() -> bool:
    return os.path.isfile(os.path.join(TARGET, "src", "train.py"))


def ensure_installed(verbose: bool = False) -> str:
    """Install the reference if it is missing; returns a one-line status."""

    if installed():
        return "present"
    src = reference_source()
    if not os.path.isdir(os.path.join(src, "src")):
        return f"reference sources not found ({src})"
    with tempfile.TemporaryDirectory(prefix="mdl_ref_") as tmp:
        copy = os.path.join(tmp, "reference")
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns("__pycache__", ".git"))
        with open(os.path.join(copy, "pyproject.toml"), "w") as fh:
            fh.write(_PYPROJECT)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", TARGET, copy]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            tail = (proc.stderr or proc.stdout).strip().splitlines()[-1:]
            return f"pip install failed: {tail}"
    if not _same_tree(os.path.join(src, "src"), os.path.join(TARGET, "src")):
        shutil.rmtree(TARGET, ignore_errors=True)
        return "installed sources differ from the reference; install removed"
    if verbose:
        print(f"reference installed under {TARGET}")
    return "installed"


if __name__ == "__main__":
    print(ensure_installed(verbose=True))
