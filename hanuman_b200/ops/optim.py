"""Fused optimizer update and gradient sum-of-squares on the native kernels."""
from __future__ import annotations

import torch

from ._ext import ext


def sumsq_cuda(bufs) -> torch.Tensor:
    out = torch.zeros(1, dtype=torch.float32, device=bufs[0].device)
    for b in bufs:
        ext().sumsq(b.contiguous(), out)
    return out.reshape(())


def fused_update_cuda(g, cfg, lr, step, coef):
    """Lion / AdamW step on a FlatGroup's shard; refreshes the working copy."""
    mode = 0 if cfg.optimizer == "adamw" else 1
    b1 = cfg.adam_b1 if mode == 0 else cfg.lion_b1
    b2 = cfg.adam_b2 if mode == 0 else cfg.lion_b2
    work = g.shard if g.sharded else g.work[g.lo:g.hi]
    ext().fused_update(g.master, g.grad[g.lo:g.hi], g.m, g.v, g.decay, work, mode, float(lr),
                       float(cfg.weight_decay), float(b1), float(b2), float(cfg.adam_eps),
                       int(step), coef.reshape(1).float().contiguous())
