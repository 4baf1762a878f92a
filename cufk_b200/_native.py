"""Loads the native extension; fails loudly when it is missing (there is no CPU fallback)."""

from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcufkb.so"

try:
    # _C.so finds libcufkb.so through its $ORIGIN run path; loading it here first also covers
    # copies of the package whose run path was stripped.
    _LIB = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    from . import _C  # noqa: E402
except OSError as exc:  # pragma: no cover - exercised only on an unbuilt checkout
    raise ImportError(
        f"cufk_b200 native library not built ({exc}); run `python cufk_b200/build.py` "
        "(or __graft_entry__.build()) first"
    ) from exc

__all__ = ["_C", "LIB_PATH"]
