"""Operator layer.

Each public function runs the hand-written sm_100a kernel when its inputs live
on a CUDA device (raising if the native extension is missing) and the pure
PyTorch math of :mod:`hanuman_b200.ops.reference` on the CPU.  The CPU path is
the execution path of the tiny fp32 configuration and the oracle of every
kernel test.

Weights are ``nn.Parameter`` fp32 masters.  When a training engine owns the
model it attaches ``p.work`` (the compute-dtype working copy) and
``p.main_grad`` (a view into the flat fp32 gradient buffer); GEMM backward
kernels accumulate weight gradients straight into ``main_grad``.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import reference as ref
from ._ext import available as ext_available  # noqa: F401
from ._ext import check_status, ext  # noqa: F401


def on_gpu(t: torch.Tensor) -> bool:
    return t.is_cuda


def working(p: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The compute-dtype copy of a parameter (engine-provided when present)."""
    w = getattr(p, "work", None)
    if w is not None and w.dtype == dtype:
        return w
    return p.detach().to(dtype)


# ------------------------------------------------------------------ linear
def linear(x: torch.Tensor, w: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
           compute_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``x @ w`` with ``w`` stored ``[in, out]`` (reference layout)."""
    if on_gpu(x):
        from .dense import linear_cuda
        return linear_cuda(x, w, out_dtype or compute_dtype, compute_dtype)
    y = x.to(compute_dtype) @ w.to(compute_dtype)
    return y if out_dtype is None else y.to(out_dtype)


def linear_t(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w^T`` in fp32 output (the tied head: ``w`` is the ``[V, D]`` embedding)."""
    if on_gpu(x):
        from .dense import linear_t_cuda
        return linear_t_cuda(x, w, torch.float32)
    return x.float() @ w.float().t()


# ------------------------------------------------------------------ norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    if on_gpu(x):
        from .norm import rms_norm_cuda
        return rms_norm_cuda(x, w, eps, out_dtype)
    return ref.rms_norm(x, w, eps, out_dtype)


# ------------------------------------------------------------------ rope
def apply_rope(q, k, cos, sin, positions=None):
    if on_gpu(q):
        from .norm import rope_cuda
        return rope_cuda(q, k, cos, sin, positions)
    return ref.apply_rope(q, k, cos, sin, positions)


# ------------------------------------------------------------------ attention
def attention(q, k, v, window: int = 0, q_offset: int = 0):
    """Causal (optionally windowed) GQA; q ``[B,S,Nq,H]``, k/v ``[B,S,Nkv,H]``."""
    if on_gpu(q):
        from .flash import flash_attention
        return flash_attention(q, k, v, window, q_offset)
    return ref.causal_attention(q, k, v, window, q_offset=q_offset)


# ------------------------------------------------------------------ swiglu
def swiglu_act(gu: torch.Tensor) -> torch.Tensor:
    """``silu(g) * u`` for ``gu = [g | u]`` along the last axis."""
    if on_gpu(gu):
        from .norm import swiglu_cuda
        return swiglu_cuda(gu)
    F = gu.shape[-1] // 2
    return torch.nn.functional.silu(gu[..., :F]) * gu[..., F:]


# ------------------------------------------------------------------ KDA
def kda_core(q, k, v, g, beta, scale: float, chunk: int, recompute: bool = False):
    """Gated delta rule over the sequence; fp32 in/out.  ``recompute`` keeps
    only the inputs for the backward (the chunk intermediates are recomputed)."""
    if on_gpu(q):
        from .kda import KdaCoreFn
        return KdaCoreFn.apply(q, k, v, g, beta, scale, recompute)
    if recompute and torch.is_grad_enabled():
        from torch.utils.checkpoint import checkpoint
        return checkpoint(lambda *a: ref.kda_chunked(*a, scale, chunk)[0], q, k, v, g, beta,
                          use_reentrant=False)
    o, _ = ref.kda_chunked(q, k, v, g, beta, scale, chunk)
    return o


# ------------------------------------------------------------------ loss
def head_cross_entropy(x: torch.Tensor, wte: torch.Tensor, targets: torch.Tensor,
                       valid: Optional[torch.Tensor] = None,
                       compute_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Mean CE of ``x @ wte^T`` against ``targets`` without materialising all
    logits on the GPU (chunked head GEMM + fused softmax-CE)."""
    if on_gpu(x):
        from .ce import head_ce_cuda
        return head_ce_cuda(x, wte, targets, valid, compute_dtype)
    logits = x.float() @ wte.float().t()
    if valid is None:
        return ref.cross_entropy(logits, targets)
    nll = torch.nn.functional.cross_entropy(logits, targets, reduction="none")
    return (nll * valid).sum() / valid.sum()
