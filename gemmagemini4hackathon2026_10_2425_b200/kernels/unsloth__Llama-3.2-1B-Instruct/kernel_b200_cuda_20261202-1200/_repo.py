"""Locate the checkout that holds the gemmagemini4hackathon2026_10_2425_b200 package, so this kernel
folder's scripts work wherever the folder sits: in the checkout, or linked into another project's
kernels/<model>/ directory (a symlink resolves back into the checkout)."""

import os
import sys
from pathlib import Path

PKG = "gemmagemini4hackathon2026_10_2425_b200"


def add_package_to_path() -> Path:
    """Put the checkout on sys.path and return it: $B2D_REPO if set, else the nearest parent of
    this file's resolved location that contains the package."""
    env = os.environ.get("B2D_REPO")
    candidates = ([Path(env)] if env else []) + list(Path(__file__).resolve().parents)
    for c in candidates:
        if (c / PKG / "__init__.py").is_file():
            if str(c) not in sys.path:
                sys.path.insert(0, str(c))
            return c
    raise SystemExit(f"cannot find the {PKG} package: set B2D_REPO to the checkout that holds it")
