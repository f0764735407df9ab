"""Loader for the in-tree CUDA extension ``carbon_b200._C`` (built by ``setup.py build_ext --inplace``).

CUDA tensors are served only by this extension: if it is missing or fails to import on a machine with a GPU, every
op raises instead of falling back to PyTorch.  CPU tensors use the fp32 oracle in ``carbon_b200.ref`` (that is the
test oracle path, not a production fallback).
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR = None


def ext():
    """Return the compiled extension module or raise a RuntimeError naming the import failure."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is None:
        try:
            import torch  # noqa: F401  (libtorch must be loaded first)

            _C = importlib.import_module("carbon_b200._C")
            return _C
        except Exception as e:  # pragma: no cover - depends on the build
            _ERR = e
    raise RuntimeError(
        "carbon_b200._C is not built or failed to load (run `python setup.py build_ext --inplace`): " + repr(_ERR))


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def so_path() -> str:
    return os.path.abspath(ext().__file__)
