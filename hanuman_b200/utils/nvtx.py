"""NVTX ranges for timeline tools (Nsight Systems, or any CUPTI consumer).

``rng(name)`` marks a host-side range around the kernels a layer or an op
enqueues.  Ranges are off unless ``HB_NVTX=1`` is set, so the training step
pays nothing for them by default.  Backward ranges of every autograd node
(including this package's custom autograd functions) come from
``torch.autograd.profiler.emit_nvtx()`` around the step.
"""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("HB_NVTX", "0") == "1"


@contextlib.contextmanager
def _range(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def rng(name: str):
    """Context manager: an NVTX range named ``name`` when HB_NVTX=1, else nothing."""
    return _range(name) if ENABLED else contextlib.nullcontext()
