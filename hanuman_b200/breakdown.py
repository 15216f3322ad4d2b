"""Analytical per-component FLOP split of one training step (breakdown.py of
the reference), scaled to a measured ms/step.

    python -m hanuman_b200.breakdown --config hybrid_1p3b --ms 1700 --batch 32

Uses the same accounting as :func:`hanuman_b200.flops.step_flops` (3 x forward,
causal / windowed attention average, KDA projections + 8*H*K*V per token) and
splits it into attention (full/SWA), KDA, dense FFN, routed experts, shared
expert, router and LM head.  The split assumes uniform efficiency; the device
profile (bench / ncu) is the ground truth for where time goes.
"""
from __future__ import annotations

import argparse

from .config import get_config
from .flops import _attn_core_flops, _kda_flops, peak_flops_per_device, step_flops


def analytical_breakdown(c, batch=None):
    D, dff, S = c.d_model, c.d_ff, c.seq_len
    Nq, Nkv, H = c.n_q_heads, c.n_kv_heads, c.head_dim
    types = c.layer_types()
    tokens = (c.batch_size if batch is None else batch) * S
    comp = {"attention (full/swa)": 0.0, "kda": 0.0, "dense ffn": 0.0, "routed experts": 0.0,
            "shared expert": 0.0, "router": 0.0, "lm head": 0.0}
    dffd = c.d_ff_shared
    for i in range(c.layers):
        if types[i] == "kda":
            comp["kda"] += _kda_flops(c, D)
        else:
            proj = 2 * D * (Nq * H + 2 * Nkv * H + Nq * H)
            comp["attention (full/swa)"] += proj + _attn_core_flops(
                S, Nq, H, c.swa_window if types[i] == "swa" else None)
        if i < c.dense_layers:
            comp["dense ffn"] += 2 * 3 * D * dffd
        else:
            comp["routed experts"] += 2 * 3 * D * dff * c.n_active
            comp["shared expert"] += 2 * 3 * D * dffd * c.n_shared_experts
            comp["router"] += 2 * D * c.n_experts
    comp["lm head"] = 2 * D * c.vocab_size
    return {k: 3 * v * tokens for k, v in comp.items()}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="hybrid_1p3b")
    ap.add_argument("--ms", type=float, default=1000.0, help="measured ms/step")
    ap.add_argument("--batch", type=int, default=None, help="sequences per step (default: config)")
    ap.add_argument("--gpus", type=int, default=1)
    a = ap.parse_args(argv)
    c = get_config(a.config)
    comps = analytical_breakdown(c, a.batch)
    model, hw = step_flops(c, a.batch)
    print(f"{'component':<24} {'TFLOP':>10} {'% step':>8} {'est. ms':>9}")
    for k, v in comps.items():
        print(f"{k:<24} {v/1e12:>10.2f} {100*v/model:>7.1f}% {v/model*a.ms:>9.1f}")
    peak = peak_flops_per_device() * a.gpus
    print(f"{'TOTAL (model)':<24} {model/1e12:>10.2f}   100.0% {a.ms:>9.1f}")
    print(f"achieved {model/1e12/(a.ms/1e3):.1f} TFLOP/s -> MFU {100*model/(a.ms/1e3)/peak:.1f}% "
          f"of {peak/1e12:.0f} TFLOP/s")


if __name__ == "__main__":
    main()
