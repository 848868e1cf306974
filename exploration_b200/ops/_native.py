"""Loader for the in-tree sm_100a extension.

The extension is compiled ahead of time by :func:`exploration_b200.build.build`
into ``exploration_b200/_build/`` and loaded from there; importing the package
never compiles. On a machine with a GPU a missing or stale extension is an
error, never a silent switch to the torch reference: every CUDA tensor that
reaches an op whose native kernel is absent raises ``NativeUnavailable``.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
from pathlib import Path

import torch

EXT_NAME = "eb200_C"
BUILD_DIR = Path(__file__).resolve().parents[1] / "_build"

_module = None
_error: str | None = None


class NativeUnavailable(RuntimeError):
    """The sm_100a extension is not built or does not load."""


def so_path() -> Path | None:
    for candidate in sorted(BUILD_DIR.glob(f"{EXT_NAME}*.so")):
        return candidate
    return None


def load(required: bool = True):
    """Return the loaded extension module (``None`` when optional and absent)."""
    global _module, _error
    if _module is not None:
        return _module
    path = so_path()
    if path is None:
        _error = f"{EXT_NAME} is not built (run `python -m exploration_b200.build`)"
    else:
        try:
            loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, str(path))
            spec = importlib.util.spec_from_file_location(EXT_NAME, str(path), loader=loader)
            module = importlib.util.module_from_spec(spec)
            loader.exec_module(module)
            _module = module
            return module
        except ImportError as exc:  # wrong torch ABI, missing symbol, ...
            _error = f"{EXT_NAME} failed to load from {path}: {exc}"
    if required:
        raise NativeUnavailable(_error)
    return None


def available() -> bool:
    return load(required=False) is not None


def native(tensor: torch.Tensor):
    """Extension for an op on ``tensor``'s device; raises for CUDA tensors if absent."""
    if not tensor.is_cuda:
        raise NativeUnavailable("native kernels run on CUDA tensors only")
    return load(required=True)

