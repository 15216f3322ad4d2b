"""Linear layers on the tcgen05 GEMM.

``linear_multi(x, [w1, w2, ...])`` runs several projections of the same input
(q/k/v, gate/up, ...) as separate GEMMs whose outputs may be column slices of
one buffer; the backward writes ONE fp32 input gradient (the later GEMMs
accumulate into it) and accumulates every weight gradient ``x^T dy`` straight
into the parameter's fp32 ``main_grad`` slice of the engine's flat buffer.
Weights are stored ``[in, out]``, so the forward is an (A K-major, B MN-major)
product, dx an (A K-major, B K-major) one and dW an (A MN-major, B MN-major)
one: no transposes are materialised.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from ._ext import ext


def _work(w: torch.Tensor) -> torch.Tensor:
    """bf16 working copy of a weight (the engine points ``w.data`` at it)."""
    if w.dtype == torch.bfloat16:
        return w.detach()
    wk = getattr(w, "_bf16_cache", None)
    if wk is None or wk._version_src != w._version:
        wk = w.detach().to(torch.bfloat16).contiguous()
        wk._version_src = w._version
        w._bf16_cache = wk
    return wk


def main_grad(w: torch.Tensor) -> torch.Tensor:
    g = getattr(w, "main_grad", None)
    if g is None:
        g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        w.main_grad = g
    return g


def _bf16(x: torch.Tensor) -> torch.Tensor:
    """bf16 2-D operand with unit column stride (row stride is kept: the TMA
    descriptors take it, so column slices of a wider buffer need no copy)."""
    x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    if x.dim() != 2 or x.stride(-1) != 1 or (x.stride(0) * 2) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


class LinearMulti(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, out_dtype, grad_dtype, *weights):
        xb = _bf16(x)
        ws = [_work(w) for w in weights]
        outs = []
        for w in ws:
            y = torch.empty(xb.shape[0], w.shape[1], dtype=out_dtype, device=x.device)
            ext().gemm(xb, w, y, False, False, False, 1.0)
            outs.append(y)
        ctx.save_for_backward(xb, *ws)
        ctx.params = weights
        ctx.grad_dtype = grad_dtype
        ctx.x_dtype = x.dtype
        return tuple(outs)

    @staticmethod
    def backward(ctx, *douts):
        xb, *ws = ctx.saved_tensors
        dx = None
        if ctx.needs_input_grad[0]:
            # one projection of a bf16 input: the GEMM writes the bf16 gradient itself
            direct = ctx.x_dtype == torch.bfloat16 and len(ws) == 1
            dx = torch.empty(xb.shape, dtype=torch.bfloat16 if direct else torch.float32,
                             device=xb.device)
        first = True
        for dy, w, p in zip(douts, ws, ctx.params):
            if dy is None:
                continue
            dyb = _bf16(dy)
            if dx is not None:
                ext().gemm(dyb, w, dx, False, True, not first, 1.0)
                first = False
            ext().gemm(xb, dyb, main_grad(p), True, False, True, 1.0)
        if dx is not None and first:
            dx.zero_()
        if dx is not None and dx.dtype != ctx.x_dtype:
            dx = dx.to(ctx.x_dtype)
        return (dx, None, None) + (None,) * len(ws)


def linear_multi(x: torch.Tensor, weights: Sequence[torch.Tensor],
                 out_dtype: torch.dtype = torch.bfloat16) -> tuple:
    return LinearMulti.apply(x, out_dtype, torch.float32, *weights)


def linear_cuda(x, w, out_dtype, compute_dtype=torch.bfloat16):
    if compute_dtype != torch.bfloat16:
        raise NotImplementedError("GPU linear layers run in bf16")
    return LinearMulti.apply(x.reshape(-1, x.shape[-1]), out_dtype, torch.float32, w)[0]


class LinearT(torch.autograd.Function):
    """``x @ w^T`` for ``w`` stored ``[out, in]`` (the tied embedding as head)."""

    @staticmethod
    def forward(ctx, x, w, out_dtype):
        xb, wb = _bf16(x), _work(w)
        y = torch.empty(xb.shape[0], wb.shape[0], dtype=out_dtype, device=x.device)
        ext().gemm(xb, wb, y, False, True, False, 1.0)
        ctx.save_for_backward(xb, wb)
        ctx.param = w
        return y

    @staticmethod
    def backward(ctx, dy):
        xb, wb = ctx.saved_tensors
        dyb = _bf16(dy)
        dx = torch.empty(xb.shape, dtype=torch.float32, device=xb.device)
        ext().gemm(dyb, wb, dx, False, False, False, 1.0)
        ext().gemm(dyb, xb, main_grad(ctx.param), True, False, True, 1.0)
        return dx, None, None


def linear_t_cuda(x, w, out_dtype=torch.float32):
    return LinearT.apply(x, w, out_dtype)


def _tma_ok(n_cols: int, elt: int = 2) -> bool:
    return (n_cols * elt) % 16 == 0


def _gemm_or_narrow(a, b, c, ta, tb, acc):
    """tcgen05 GEMM, or (only for widths TMA cannot address: fewer than 8 bf16
    columns, as in the tiny smoke presets) an fp32 matmul of the same product."""
    if all(_tma_ok(t.shape[1]) and _tma_ok(t.stride(0)) for t in (a, b)) and \
            _tma_ok(c.stride(0), c.element_size()):
        ext().gemm(a, b, c, ta, tb, acc, 1.0)
        return
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    r = A @ B
    if acc:
        c.add_(r.to(c.dtype))
    else:
        c.copy_(r.to(c.dtype))


class LinearFused(torch.autograd.Function):
    """Several projections of one input written side by side into ONE output
    ``[T, sum(N_i)]`` (column slices), e.g. q|k|v.  Backward reads the column
    slices of the output gradient in place (strided TMA rows, no copies)."""

    @staticmethod
    def forward(ctx, x, out_dtype, *weights):
        xb = _bf16(x)
        ws = [_work(w) for w in weights]
        ntot = sum(w.shape[1] for w in ws)
        y = torch.empty(xb.shape[0], ntot, dtype=out_dtype, device=x.device)
        off = 0
        for w in ws:
            _gemm_or_narrow(xb, w, y[:, off:off + w.shape[1]], False, False, False)
            off += w.shape[1]
        ctx.save_for_backward(xb, *ws)
        ctx.params = weights
        ctx.x_dtype = x.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        xb, *ws = ctx.saved_tensors
        dyb = _bf16(dy)
        direct = ctx.x_dtype == torch.bfloat16 and len(ws) == 1
        dx = torch.empty(xb.shape, dtype=torch.bfloat16 if direct else torch.float32,
                         device=xb.device) if ctx.needs_input_grad[0] else None
        off = 0
        for i, (w, p) in enumerate(zip(ws, ctx.params)):
            sl = dyb[:, off:off + w.shape[1]]
            if dx is not None:
                _gemm_or_narrow(sl, w, dx, False, True, i > 0)
            _gemm_or_narrow(xb, sl, main_grad(p), True, False, True)
            off += w.shape[1]
        if dx is not None and dx.dtype != ctx.x_dtype:
            dx = dx.to(ctx.x_dtype)
        return (dx, None) + (None,) * len(ws)


def linear_fused(x: torch.Tensor, weights: Sequence[torch.Tensor],
                 out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    return LinearFused.apply(x, out_dtype, *weights)
