"""Checkpoint save / resume and export to the reference parameter tree.

Layout of ``<checkpoint_dir>/<name>/step_<N>/``:

    params.safetensors   fp32 master weights, keys = reference tree names
                         (``blocks/0/attn/wq``), shapes = reference shapes
    optim_rank<r>.pt     this rank's optimizer-state shards
    extra_rank<r>.pt     per-rank extras (data-loader RNG state)
    meta.json            step, world size, config

Writes go to ``step_<N>.tmp`` and are renamed into place, so a crash never
leaves a half-written checkpoint that ``latest_checkpoint`` would pick.  The
reference saves params only, at the end of a run (train.py:326-334); this
adds optimizer + loader state and periodic saves (``checkpoint_every``).
``export_reference_tree`` restacks block parameters into the reference's
scan-path layout (``moe_stack/blocks/...`` with a leading layer axis) when the
configuration would use the scan path (model/transformer.py:314-358).
"""
from __future__ import annotations

import json
import os
import shutil
from dataclasses import asdict

import torch


def ref_name(name: str) -> str:
    return name.replace(".", "/")


def from_ref_name(name: str) -> str:
    return name.replace("/", ".")


def param_shapes(config) -> dict:
    """{dotted name: shape} of the model for ``config`` without allocating."""
    from .models import layers
    from .models.transformer import Transformer
    layers._META = True
    try:
        with torch.device("meta"):
            m = Transformer(config)
    finally:
        layers._META = False
    return {n: tuple(p.shape) for n, p in m.named_parameters()}


def _ckpt_dir(config):
    return os.path.abspath(os.path.join(config.checkpoint_dir, config.name))


def latest_checkpoint(config):
    d = _ckpt_dir(config)
    if not os.path.isdir(d):
        return None
    steps = [s for s in os.listdir(d) if s.startswith("step_") and not s.endswith(".tmp")
             and os.path.exists(os.path.join(d, s, "meta.json"))]
    if not steps:
        return None
    steps.sort(key=lambda s: int(s.split("_")[1]))
    return os.path.join(d, steps[-1])


def save_checkpoint(trainer, config, step: int, dist_ctx=None, extra=None):
    from safetensors.torch import save_file
    rank = dist_ctx.rank if dist_ctx else 0
    world = dist_ctx.world if dist_ctx else 1
    params = trainer.engine.master_state()   # collective under data parallelism
    final = os.path.join(_ckpt_dir(config), f"step_{step}")
    tmp = final + ".tmp"
    if rank == 0:
        if os.path.exists(tmp):
            shutil.rmtree(tmp)
        os.makedirs(tmp, exist_ok=True)
    if dist_ctx is not None and world > 1:
        dist_ctx.barrier()
    if rank == 0:
        save_file({ref_name(k): v.detach().float().cpu().contiguous() for k, v in params.items()},
                  os.path.join(tmp, "params.safetensors"))
    opt = {k: {kk: vv.cpu() for kk, vv in d.items()} for k, d in trainer.engine.optimizer_state().items()}
    torch.save(opt, os.path.join(tmp, f"optim_rank{rank}.pt"))
    torch.save(extra or {}, os.path.join(tmp, f"extra_rank{rank}.pt"))
    if dist_ctx is not None and world > 1:
        dist_ctx.barrier()
    if rank == 0:
        with open(os.path.join(tmp, "meta.json"), "w") as f:
            json.dump({"step": step, "world": world, "config": asdict(config)}, f, indent=1)
        if os.path.exists(final):
            shutil.rmtree(final)
        os.replace(tmp, final)
        print(f"[train] Saved checkpoint to {final}")
    if dist_ctx is not None and world > 1:
        dist_ctx.barrier()
    return final


def load_params(path) -> dict:
    from safetensors.torch import load_file
    st = load_file(os.path.join(path, "params.safetensors"))
    return {from_ref_name(k): v for k, v in st.items()}


def load_checkpoint(trainer, path, dist_ctx=None) -> dict:
    """Restore params, optimizer shards and step; returns this rank's extras."""
    rank = dist_ctx.rank if dist_ctx else 0
    with open(os.path.join(path, "meta.json")) as f:
        meta = json.load(f)
    params = load_params(path)
    shapes = {n: tuple(p.shape) for n, p in trainer.model.named_parameters()}
    missing = set(shapes) - set(params)
    if missing:
        raise KeyError(f"checkpoint {path} lacks {sorted(missing)[:5]}")
    for n, s in shapes.items():
        if tuple(params[n].shape) != s:
            raise ValueError(f"shape mismatch for {n}: {tuple(params[n].shape)} vs {s}")
    trainer.engine.load_master_state(params)
    opt_file = os.path.join(path, f"optim_rank{rank}.pt")
    world = dist_ctx.world if dist_ctx else 1
    if os.path.exists(opt_file) and meta.get("world", 1) == world:
        trainer.engine.load_optimizer_state(torch.load(opt_file, map_location="cpu"))
    trainer.engine.step_count = int(meta["step"])
    ex = os.path.join(path, f"extra_rank{rank}.pt")
    return torch.load(ex, weights_only=False) if os.path.exists(ex) else {}


def export_reference_tree(params: dict, config) -> dict:
    """Map our dotted names to the reference's tree paths.

    KDA hybrids (and ``use_scan=False``) use the loop layout
    ``blocks/<i>/...``; otherwise blocks are stacked on a leading layer axis
    under ``dense_stack/blocks`` and ``moe_stack/blocks``.
    """
    use_scan = config.use_scan and not config.use_kda
    out = {}
    if not use_scan:
        for k, v in params.items():
            out[ref_name(k)] = v
        return out
    per_layer = {}
    for k, v in params.items():
        if k.startswith("blocks."):
            _, i, rest = k.split(".", 2)
            per_layer.setdefault(rest, {})[int(i)] = v
        else:
            out[ref_name(k)] = v
    nd = config.dense_layers
    for rest, by_layer in per_layer.items():
        dense = [by_layer[i] for i in range(nd) if i in by_layer]
        moe = [by_layer[i] for i in range(nd, config.layers) if i in by_layer]
        if dense:
            out["dense_stack/blocks/" + ref_name(rest)] = torch.stack(dense)
        if moe:
            out["moe_stack/blocks/" + ref_name(rest)] = torch.stack(moe)
    return out
