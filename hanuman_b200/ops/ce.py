"""Tied LM head fused with softmax cross-entropy (train.py:186-196).

The head GEMM runs over token chunks.  Each chunk's fp32 logits are consumed
at once by the CE kernel, which writes the chunk's loss contribution and its
bf16 gradient ``(softmax - onehot) / N``; that gradient then feeds the chunk's
two head-backward GEMMs right away (``dx`` rows, and ``dW`` accumulated in
fp32) and is overwritten by the next chunk.  Neither the logits nor their
gradient ever exist for all ``T x V`` at once: the forward keeps ``dx``
``[T, D]`` and ``dW`` ``[V, D]`` (fp32), and the backward scales them by the
incoming gradient (a device scalar) into the input gradient and the weight's
gradient accumulator.  Without autograd (evaluation) only the loss is computed.
"""
from __future__ import annotations

import torch

from ._ext import ext
from .dense import _bf16, _work, main_grad

CHUNK_TOKENS = 4096


class HeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, targets, valid):
        xb = _bf16(x)
        wb = _work(w)
        T, D = xb.shape
        V = wb.shape[0]
        dev = x.device
        grads = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        denom = torch.tensor(float(T), device=dev) if valid is None else valid.sum().float()
        inv = (1.0 / denom).reshape(1).float().contiguous()
        loss_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        C = min(T, CHUNK_TOKENS)
        logits = torch.empty(C, V, dtype=torch.float32, device=dev)
        dlog = torch.empty(C, V, dtype=torch.bfloat16, device=dev)
        tgt = targets.reshape(-1).long().contiguous()
        vf = None if valid is None else valid.float().contiguous()
        dx = torch.empty(T, D, dtype=torch.float32, device=dev) if grads else None
        dw = torch.empty(V, D, dtype=torch.float32, device=dev) if grads else None
        for i, t0 in enumerate(range(0, T, C)):
            t1 = min(T, t0 + C)
            n = t1 - t0
            lg, dl = logits[:n], dlog[:n]
            ext().gemm(xb[t0:t1], wb, lg, False, True, False, 1.0)
            # chunk gradient (softmax - onehot) [* valid]; the 1/N of the mean
            # enters the two GEMMs below as a device-side alpha
            ext().ce_fwd_bwd(lg, tgt[t0:t1], None if vf is None else vf[t0:t1], loss_sum, dl, 1.0)
            if grads:
                ext().gemm(dl, wb, dx[t0:t1], False, False, False, 1.0, inv)
                ext().gemm(dl, xb[t0:t1], dw, True, False, i > 0, 1.0, inv)
        del logits, dlog
        if grads:
            ctx.save_for_backward(dx, dw)
        ctx.param = w
        return (loss_sum / denom).reshape(())

    @staticmethod
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        gs = g.float().reshape(1)
        dx.mul_(gs)
        mg = main_grad(ctx.param)
        mg.addcmul_(dw, gs.to(mg.dtype)) if mg.dtype == dw.dtype else mg.add_((dw * gs).to(mg.dtype))
        return dx, None, None, None


def head_ce_cuda(x, w, targets, valid=None, compute_dtype=torch.bfloat16):
    return HeadCEFn.apply(x, w, targets, valid)
