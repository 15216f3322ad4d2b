"""Parameter counts, FLOP accounting and MFU (train.py:29-177 of the reference).

``step_flops`` keeps the reference's conventions so that MFU numbers are
comparable: model FLOPs = 3 x forward; attention core 4*Nq*H*avg_keys with the
causal / sliding-window average; KDA = projections + 8*H*K*V per token for the
recurrence; hardware FLOPs add one block forward when remat is on.
"""
from __future__ import annotations

import json
import os
from typing import Optional

from .config import Config


def count_active_params(c: Config) -> int:
    D, dff = c.d_model, c.d_ff
    emb = c.vocab_size * D
    attn = D * (c.n_q_heads * c.head_dim) + 2 * D * (c.n_kv_heads * c.head_dim) \
        + (c.n_q_heads * c.head_dim) * D
    dffd = c.d_ff_shared
    dense_ffn = 3 * D * dffd
    moe_active = c.n_active * 3 * D * dff + c.n_shared_experts * 3 * D * dffd
    router = D * c.n_experts
    n_dense = c.dense_layers
    n_moe = c.layers - n_dense
    return (emb + n_dense * (attn + dense_ffn + 2 * D) + n_moe * (attn + moe_active + 2 * D)
            + 3 * D + c.layers + router)


def count_total_params(c: Config) -> int:
    D, dff = c.d_model, c.d_ff
    emb = c.vocab_size * D
    attn = D * (c.n_q_heads * c.head_dim) + 2 * D * (c.n_kv_heads * c.head_dim) \
        + (c.n_q_heads * c.head_dim) * D
    dffd = c.d_ff_shared
    dense_ffn = 3 * D * dffd
    moe_total = c.n_experts * 3 * D * dff + c.n_shared_experts * 3 * D * dffd
    n_dense = c.dense_layers
    n_moe = c.layers - n_dense
    return (emb + n_dense * (attn + dense_ffn + 2 * D) + n_moe * (attn + moe_total + 2 * D)
            + 3 * D + c.layers + D * c.n_experts + c.n_experts)


def count_model_params(model) -> int:
    return sum(p.numel() for p in model.parameters())


def _attn_core_flops(S: int, Nq: int, H: int, window: Optional[int]) -> float:
    if not window or window >= S:
        avg = (S + 1) / 2
    else:
        W = float(window)
        avg = (W * (W + 1) / 2 + (S - W) * W) / S
    return 4 * Nq * H * avg


def _kda_flops(c: Config, D: int) -> float:
    Hk, Kd = c.kda_heads, c.kda_head_dim
    V = Kd
    proj = 2 * D * (3 * Hk * Kd)
    proj += 2 * D * Kd + 2 * Kd * (Hk * Kd)
    proj += 2 * D * Kd + 2 * Kd * (Hk * V)
    proj += 2 * D * Hk
    proj += 2 * (Hk * V) * D
    return proj + 8 * Hk * Kd * V


def step_flops(c: Config, batch: Optional[int] = None) -> tuple[int, int]:
    """(model_flops, hardware_flops) for one optimizer step of ``batch`` sequences."""
    D, dff, S = c.d_model, c.d_ff, c.seq_len
    Nq, Nkv, H = c.n_q_heads, c.n_kv_heads, c.head_dim
    types = c.layer_types()

    def layer_attn(i):
        if types[i] == "kda":
            return _kda_flops(c, D)
        proj = 2 * D * (Nq * H + 2 * Nkv * H + Nq * H)
        return proj + _attn_core_flops(S, Nq, H, c.swa_window if types[i] == "swa" else None)

    dffd = c.d_ff_shared
    dense_ffn = 2 * 3 * D * dffd
    moe_ffn = 2 * 3 * D * (dff * c.n_active + dffd * c.n_shared_experts)
    router = 2 * D * c.n_experts
    head = 2 * D * c.vocab_size
    block_fwd = 0.0
    for i in range(c.layers):
        block_fwd += layer_attn(i) + (dense_ffn if i < c.dense_layers else moe_ffn + router)
    tokens = (c.batch_size if batch is None else batch) * S
    model = 3 * (block_fwd + head) * tokens
    hw = model + (block_fwd * tokens if c.remat else 0)
    return int(model), int(hw)


def peak_flops_per_device() -> float:
    """Measured bf16 peak of this pool's B200 (MEASURED_PEAKS.json next to the
    repository root), else NVIDIA's dense bf16 figure."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = os.path.join(here, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]) * 1e12
    except Exception:
        return 2.25e15
