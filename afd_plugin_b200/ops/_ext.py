"""Loader for the in-tree sm_100a extension (``afd_plugin_b200/_C*.so``).

The library registers its kernels as ``torch.ops.afd_b200.*``.  On a CUDA
tensor every op goes to the extension; if the library was not built the call
raises instead of silently running something else.
"""

from __future__ import annotations

import glob
import os
import threading

import torch

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_lock = threading.Lock()
_loaded_path: str | None = None
_load_error: str | None = None


def library_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(_PKG_DIR, "_C*.so")))
    return hits[0] if hits else None


def load() -> bool:
    """Load the extension once; return whether it is available."""
    global _loaded_path, _load_error
    if _loaded_path is not None:
        return True
    with _lock:
        if _loaded_path is not None:
            return True
        path = library_path()
        if path is None:
            _load_error = "afd_plugin_b200/_C*.so not found: run `python setup.py build_ext --inplace`"
            return False
        try:
            torch.ops.load_library(path)
        except OSError as exc:  # pragma: no cover - depends on the box
            _load_error = f"failed to load {path}: {exc}"
            return False
        _loaded_path = path
        return True


def ops():
    """``torch.ops.afd_b200`` namespace; raises if the extension is missing."""
    if not load():
        raise RuntimeError(f"afd_b200 CUDA extension unavailable: {_load_error}")
    return torch.ops.afd_b200


def loaded_path() -> str | None:
    return _loaded_path


__all__ = ["library_path", "load", "loaded_path", "ops"]
