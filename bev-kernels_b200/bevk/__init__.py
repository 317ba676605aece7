"""Runtime helpers of the B200 deformable-sampling kernels.

* :mod:`bevk.cabi` -- ctypes binding of ``libbevk.so`` (the C ABI declared in
  ``include/bevk.h``); usable without the torch extensions.
* :func:`load_extension` -- imports a torch extension built next to this
  package, failing loudly (there is no CPU or eager fallback).
"""
from __future__ import annotations

import importlib
import os

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_ROOT, "libbevk.so")

_BUILD_HINT = "build it with `python bev-kernels_b200/build.py` (nvcc, sm_100a)"


def load_extension(name: str):
    """Import the in-tree torch extension ``name`` or raise ImportError."""
    try:
        return importlib.import_module(name)
    except ImportError as e:  # pragma: no cover - exercised when unbuilt
        raise ImportError(f"bev-kernels_b200: extension {name} is not available ({e}); "
                          f"{_BUILD_HINT}") from e
