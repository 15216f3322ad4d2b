"""Tied LM head fused with softmax cross-entropy (train.py:186-196).

The head GEMM runs over token chunks; each chunk's fp32 logits are consumed
immediately by the CE kernel, which writes the chunk's loss contribution and
its bf16 gradient ``(softmax - onehot) / N``.  The full fp32 ``[T, V]`` logits
never exist; the backward multiplies by the incoming gradient on the device
(GEMM alpha read from device memory) and runs the two head GEMMs.
"""
from __future__ import annotations

import torch

from ._ext import ext
from .dense import _bf16, _work, main_grad

CHUNK_TOKENS = 8192


class HeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, targets, valid):
        xb = _bf16(x)
        wb = _work(w)
        T = xb.shape[0]
        V = wb.shape[0]
        n = float(T) if valid is None else None
        denom = torch.tensor(float(T), device=x.device) if valid is None else valid.sum()
        loss_sum = torch.zeros(1, dtype=torch.float32, device=x.device)
        dlogits = torch.empty(T, V, dtype=torch.bfloat16, device=x.device)
        logits = torch.empty(min(T, CHUNK_TOKENS), V, dtype=torch.float32, device=x.device)
        tgt = targets.reshape(-1).long().contiguous()
        vf = None if valid is None else valid.float().contiguous()
        scale = 1.0 / n if n is not None else 1.0
        for t0 in range(0, T, CHUNK_TOKENS):
            t1 = min(T, t0 + CHUNK_TOKENS)
            lg = logits[: t1 - t0]
            ext().gemm(xb[t0:t1], wb, lg, False, True, False, 1.0)
            ext().ce_fwd_bwd(lg, tgt[t0:t1], None if vf is None else vf[t0:t1], loss_sum,
                             dlogits[t0:t1], scale)
        if valid is not None:
            dlogits.div_(denom.to(torch.bfloat16))
        ctx.save_for_backward(xb, wb, dlogits)
        ctx.param = w
        return (loss_sum / denom).reshape(())

    @staticmethod
    def backward(ctx, g):
        xb, wb, dlogits = ctx.saved_tensors
        gs = g.float().reshape(1).contiguous()
        dx = torch.empty(xb.shape, dtype=torch.float32, device=xb.device)
        ext().gemm(dlogits, wb, dx, False, False, False, 1.0, gs)
        ext().gemm(dlogits, xb, main_grad(ctx.param), True, False, True, 1.0, gs)
        return dx, None, None, None


def head_ce_cuda(x, w, targets, valid=None, compute_dtype=torch.bfloat16):
    return HeadCEFn.apply(x, w, targets, valid)
