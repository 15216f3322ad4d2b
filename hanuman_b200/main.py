"""Command line: ``train | generate | count | report`` (main.py:150-235).

    python main.py train --config smoke
    python main.py train --config hybrid_1p3b --steps 100
    torchrun --nproc-per-node 8 main.py train --config hybrid_1p3b
    python main.py generate --config smoke --prompt "hello" --max_tokens 20
    python main.py count --config full
    python main.py report --config full_g4
"""
from __future__ import annotations

import argparse


def _apply_overrides(config, args):
    mapping = {
        "steps": "train_steps", "batch": "batch_size", "seq_len": "seq_len", "remat": "remat",
        "remat_policy": "remat_policy", "experts": "n_experts", "d_ff": "d_ff",
        "d_ff_dense": "d_ff_dense", "n_active": "n_active", "dense_layers": "dense_layers",
        "z_weight": "z_loss_weight", "bias_rate": "bias_update_rate",
        "balance_weight": "balance_loss_weight", "warmup": "warmup_steps", "lr": "learning_rate",
        "log_every": "log_every", "data_axis": "mesh_data_axis", "expert_axis": "mesh_expert_axis",
        "use_swa": "use_swa", "swa_window": "swa_window", "swa_period": "swa_period",
        "use_grain": "use_grain", "gen_every": "gen_every", "gen_prompt": "gen_prompt",
        "gen_max_tokens": "gen_max_tokens", "use_kda": "use_kda", "kda_period": "kda_period",
        "optimizer": "optimizer", "router_type": "router_type",
        "capacity_factor": "capacity_factor", "micro_batch": "micro_batch",
        "checkpoint_every": "checkpoint_every", "fused_comm": "fused_comm",
        "expert_weights": "expert_weights", "metrics_jsonl": "metrics_jsonl",
    }
    for a, f in mapping.items():
        v = getattr(args, a, None)
        if v is not None:
            setattr(config, f, v)
    return config


def cmd_train(args):
    from .config import get_config
    from .parallel.mesh import init_distributed
    from .train import train
    config = _apply_overrides(get_config(args.config), args)
    ctx = init_distributed()
    try:
        train(config, use_random_data=True, save=not args.no_save, dist_ctx=ctx,
              resume=args.resume)
    finally:
        if ctx is not None:
            ctx.shutdown()


def cmd_generate(args):
    from .config import get_config
    from .generate import load_for_generate
    config = get_config(args.config)
    if args.yarn_factor is not None:
        config.yarn_factor = args.yarn_factor
    text, ids = load_for_generate(config, args.prompt, args.max_tokens, args.temperature,
                                  args.top_k, args.seed, cached=args.cache)
    print("=== Generated ===")
    print(text)
    print("=== Token ids ===")
    print(ids)


def cmd_count(args):
    from .config import get_config
    from .flops import count_active_params, count_total_params
    c = get_config(args.config)
    total, active = count_total_params(c), count_active_params(c)
    print(f"Config: {c.name}")
    print(f"  Layers: {c.layers} (dense={c.dense_layers}, moe={c.layers - c.dense_layers}) "
          f"types={c.layer_types()}")
    print(f"  d_model={c.d_model}, d_ff={c.d_ff}, heads q/kv={c.n_q_heads}/{c.n_kv_heads} "
          f"head_dim={c.head_dim}")
    print(f"  Experts: {c.n_experts} routed + {c.n_shared_experts} shared, top-{c.n_active}")
    print(f"  Total params:   {total:,} ({total/1e9:.3f}B)")
    print(f"  Active params:  {active:,} ({active/1e9:.3f}B)")


def cmd_report(args):
    from .config import get_config
    from .train import memory_report
    print(memory_report(get_config(args.config)))


def build_parser():
    from .config import PRESETS
    p = argparse.ArgumentParser(description="hanuman_b200 hybrid MoE transformer")
    sub = p.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("train", help="Run training")
    t.add_argument("--config", default="full_g4", choices=list(PRESETS))
    for name, typ in [("steps", int), ("batch", int), ("seq_len", int), ("experts", int),
                      ("d_ff", int), ("d_ff_dense", int), ("n_active", int),
                      ("dense_layers", int), ("z_weight", float), ("bias_rate", float),
                      ("balance_weight", float), ("warmup", int), ("lr", float),
                      ("log_every", int), ("data_axis", int), ("expert_axis", int),
                      ("swa_window", int), ("swa_period", int), ("gen_every", int),
                      ("gen_prompt", str), ("gen_max_tokens", int), ("kda_period", int),
                      ("capacity_factor", float), ("micro_batch", int),
                      ("checkpoint_every", int), ("metrics_jsonl", str)]:
        t.add_argument(f"--{name}", type=typ, default=None)
    t.add_argument("--remat_policy", default=None,
                   choices=["full", "dots", "dots_no_batch", "experts", "none"])
    t.add_argument("--optimizer", default=None, choices=["lion", "adamw"])
    t.add_argument("--router_type", default=None, choices=["sigmoid_bias", "softmax"])
    t.add_argument("--expert_weights", default=None, choices=["replicated", "fused_gather"])
    t.add_argument("--random_data", action="store_true")
    t.add_argument("--no_save", action="store_true")
    t.add_argument("--resume", action="store_true", help="continue from the latest checkpoint")
    for flag in ("remat", "use_swa", "use_grain", "use_kda", "fused_comm"):
        t.add_argument(f"--{flag}", dest=flag, action="store_true", default=None)
        t.add_argument(f"--no_{flag.replace('use_', '')}", dest=flag, action="store_false")
    t.set_defaults(func=cmd_train)
    g = sub.add_parser("generate", help="Generate text")
    g.add_argument("--config", default="smoke", choices=list(PRESETS))
    g.add_argument("--prompt", default="Once upon a time")
    g.add_argument("--max_tokens", type=int, default=100)
    g.add_argument("--temperature", type=float, default=1.0)
    g.add_argument("--top_k", type=int, default=0)
    g.add_argument("--seed", type=int, default=0)
    g.add_argument("--yarn_factor", type=float, default=None)
    g.add_argument("--cache", action="store_true",
                   help="incremental decoding with KV / KDA-state caches (same tokens, no recompute)")
    g.set_defaults(func=cmd_generate)
    c = sub.add_parser("count", help="Print param counts")
    c.add_argument("--config", default="full_g4", choices=list(PRESETS))
    c.set_defaults(func=cmd_count)
    r = sub.add_parser("report", help="Per-tensor sharding and HBM table")
    r.add_argument("--config", default="full_g4", choices=list(PRESETS))
    r.set_defaults(func=cmd_report)
    return p


def main(argv=None):
    args = build_parser().parse_args(argv)
    args.func(args)


if __name__ == "__main__":
    main()
