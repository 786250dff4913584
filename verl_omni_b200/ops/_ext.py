"""Loader for the in-tree sm_100a CUDA extension (``verl_omni_b200/_C*.so``).

CUDA tensors always go through the extension: if it is missing on a machine with a GPU the
first op raises instead of silently running a PyTorch fallback.  CPU tensors (the gloo/CPU
plumbing path and the fp32 oracles) never touch it.
"""

from __future__ import annotations

import importlib
import os

_EXT = None
_ERR: Exception | None = None


def ext():
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    if _ERR is not None:
        raise RuntimeError(f"verl_omni_b200 CUDA extension unavailable: {_ERR}") from _ERR
    try:
        import torch  # noqa: F401  (libtorch must be loaded before the extension)

        _EXT = importlib.import_module("verl_omni_b200._C")
    except Exception as e:  # pragma: no cover - only on a broken build
        _ERR = e
        raise RuntimeError(
            "verl_omni_b200 CUDA extension is not built; run `python setup.py build_ext --inplace` "
            f"(or __graft_entry__.build()): {e}") from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def so_path() -> str | None:
    try:
        return os.path.abspath(ext().__file__)
    except RuntimeError:
        return None
