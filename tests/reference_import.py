"""Locates the reference package (``DWDP``) for the tests that plug into it: the copy
staged under oracle/_ref (it travels with the repository) or the reference tree itself."""
from __future__ import annotations

import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
CANDIDATES = [ROOT / "oracle" / "_ref", pathlib.Path("/root/reference")]


def import_reference():
    """Returns the imported ``DWDP`` package, or None when no copy is present."""
    for c in CANDIDATES:
        if (c / "DWDP").is_dir():
            if str(c) not in sys.path:
                sys.path.insert(0, str(c))
            try:
                import DWDP
            except Exception:  # pragma: no cover - a broken copy counts as absent
                return None
            return DWDP
    return None
