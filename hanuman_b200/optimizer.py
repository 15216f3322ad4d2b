"""Optimizer: WSD schedule, global-norm clipping, Lion or AdamW with
learning-rate-scaled decoupled weight decay and the reference's no-decay mask.

Semantics follow optimizer.py:10-155 of the reference:
  * ``wsd_schedule``: linear warmup 0 -> lr over ``max(1, warmup)`` steps,
    constant, then cosine to ``min_lr`` over the last ``decay_fraction``;
    ``stable_steps = max(1, ...)`` (optimizer.py:18-20);
  * clip by global norm (optax ``clip_by_global_norm``);
  * Lion (b1 .9, b2 .99, momentum stored in ``opt_state_dtype``), then the
    decoupled decay ``u -= lr(t) * wd * p`` on masked leaves (optimizer.py:96-123);
  * AdamW (bias-corrected, same decay rule) for the BASELINE configurations.
The functions operating on flat tensors are the CPU implementation and the
oracle of the fused CUDA update kernel.
"""
from __future__ import annotations

import math

import torch


def wsd_lr(step: int, learning_rate: float, min_lr: float, warmup_steps: int,
           total_steps: int, decay_fraction: float) -> float:
    """Learning rate at ``step`` (0-based count of updates already applied)."""
    decay_steps = int(total_steps * decay_fraction)
    stable_steps = max(1, total_steps - warmup_steps - decay_steps)
    decay_start = warmup_steps + stable_steps
    if step < warmup_steps:
        return learning_rate * min(1.0, step / max(1, warmup_steps))
    if step < decay_start:
        return learning_rate
    t = min(step - decay_start, max(1, decay_steps))
    d = max(1, decay_steps)
    alpha = (min_lr / learning_rate) if learning_rate > 0 else 0.0
    cos = 0.5 * (1 + math.cos(math.pi * t / d))
    return learning_rate * ((1 - alpha) * cos + alpha)


def schedule_for(cfg):
    return lambda step: wsd_lr(step, cfg.learning_rate, cfg.min_lr, cfg.warmup_steps,
                               cfg.train_steps, cfg.decay_fraction)


def is_no_decay(name: str) -> bool:
    """Reference rule (optimizer.py:42-67), applied to our dotted names."""
    n = name.lower()
    return any(s in n for s in ("norm", "residual_scale", "bias", "wte", "embed", "router",
                                "cos", "sin", "a_log", "dt_bias"))


def clip_coef(grad_sq_sum: torch.Tensor, max_norm: float) -> torch.Tensor:
    """Multiplier applied to every gradient (optax clip_by_global_norm)."""
    norm = torch.sqrt(grad_sq_sum)
    return torch.where(norm < max_norm, torch.ones_like(norm), max_norm / norm)


@torch.no_grad()
def lion_update_(p, g, m, decay_mask, lr, wd, b1, b2, coef):
    """In-place Lion step on flat fp32 ``p``; ``m`` may be bf16."""
    gg = g * coef
    mf = m.float()
    u = torch.sign((1 - b1) * gg + b1 * mf)
    m.copy_((b2 * mf + (1 - b2) * gg).to(m.dtype))
    upd = -lr * u - lr * wd * p * decay_mask
    p.add_(upd)


@torch.no_grad()
def adamw_update_(p, g, m, v, decay_mask, lr, wd, b1, b2, eps, step, coef):
    """In-place AdamW step (bias-corrected; ``step`` counts from 1)."""
    gg = g * coef
    m.mul_(b1).add_((1 - b1) * gg)
    v.mul_(b2).add_((1 - b2) * gg * gg)
    mh = m / (1 - b1 ** step)
    vh = v / (1 - b2 ** step)
    upd = -lr * (mh / (vh.sqrt() + eps)) - lr * wd * p * decay_mask
    p.add_(upd)
