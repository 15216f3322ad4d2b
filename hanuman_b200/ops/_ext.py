"""Loader of the compiled sm_100a extension.

The extension is imported from the in-tree build directory.  CUDA code paths
call :func:`ext` which raises if the extension is missing, so a GPU run never
silently falls back to eager PyTorch.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys

from .. import _build

_mod = None
_err = None


def _load():
    global _mod, _err
    if _mod is not None or _err is not None:
        return
    path = _build.so_path()
    if not os.path.exists(path):
        _err = f"native extension not built ({path} missing); run `python -m hanuman_b200._build`"
        return
    try:
        import torch  # noqa: F401  (the extension links against libtorch)
        loader = importlib.machinery.ExtensionFileLoader(_build.EXT_NAME, path)
        spec = importlib.util.spec_from_file_location(_build.EXT_NAME, path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules[_build.EXT_NAME] = mod
        _mod = mod
    except Exception as e:  # pragma: no cover - surfaced through ext()
        _err = f"failed to load native extension {path}: {e!r}"


def available() -> bool:
    _load()
    return _mod is not None


def ext():
    """The loaded extension module; raises RuntimeError when unavailable."""
    _load()
    if _mod is None:
        raise RuntimeError(_err)
    return _mod


def check_status():
    """Raise if any kernel recorded a bounded-wait timeout or bounds error."""
    s = ext().read_status()
    if s != 0:
        ext().clear_status()
        raise RuntimeError(f"hanuman_b200 kernel reported error status {s}")
