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


_STATUS_NAMES = {1: "TMA producer wait timed out", 2: "MMA wait timed out",
                 3: "epilogue wait timed out", 4: "peer wait timed out",
                 5: "index out of bounds", 6: "expert capacity exceeded"}


class KernelStatusError(RuntimeError):
    """A kernel recorded an error in the device status word (a bounded wait
    that ran out of budget, a bounds check); the step that saw it is not valid."""

    def __init__(self, code: int):
        self.code = int(code)
        super().__init__(f"hanuman_b200 kernel error status {code} "
                         f"({_STATUS_NAMES.get(int(code), 'unknown')})")


class StatusMonitor:
    """Checks the device status word once per training step without stalling
    the device.

    ``poll()`` enqueues an asynchronous copy of the status word into pinned
    host memory (after the step's kernels, on the current stream) and checks
    the copy enqueued by the previous ``poll()``, waiting for that copy's
    event: the host then runs at most one step ahead of the device, and an
    error is raised at the end of the step after the one that recorded it.
    ``flush()`` waits for and checks the latest copy."""

    def __init__(self):
        self._view = ext().status_view()
        self._bufs = [torch_empty_pinned_int() for _ in range(2)]
        self._events = [None, None]
        self._i = 0

    def _check(self, j):
        ev = self._events[j]
        if ev is None:
            return
        ev.synchronize()
        self._events[j] = None
        code = int(self._bufs[j][0])
        if code != 0:
            raise KernelStatusError(code)

    def poll(self):
        import torch
        i = self._i
        self._bufs[i].copy_(self._view, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._events[i] = ev
        self._i = i ^ 1
        self._check(i ^ 1)

    def flush(self):
        self._check(self._i ^ 1)


def torch_empty_pinned_int():
    import torch
    return torch.zeros(1, dtype=torch.int32, pin_memory=True)
