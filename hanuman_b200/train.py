"""Training driver: the ``Trainer`` public API and the ``train`` loop
(train.py:398-562 of the reference).

``Trainer.step(tokens)`` is the call a user makes: it takes one global-batch
shard of token ids (host or device tensor), copies it to the device, runs the
micro-batched forward/backward, the data-parallel gradient reduction, global
norm clipping, the fused optimizer update and the router-bias update, and
returns the loss as a device tensor (``float(loss)`` reads it back).
"""
from __future__ import annotations

import json
import os
import time
from typing import Optional

import torch

from . import flops as fl
from .config import Config
from .engine import Engine
from .models.transformer import Transformer
from .utils.nvtx import rng


class Trainer:
    def __init__(self, cfg: Config, device: Optional[str] = None, seed: Optional[int] = None,
                 dist_ctx=None):
        self.cfg = cfg
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        self.dist = dist_ctx
        world = dist_ctx.world if dist_ctx is not None else 1
        rank = dist_ctx.rank if dist_ctx is not None else 0
        ep = None
        if dist_ctx is not None and world > 1 and cfg.mesh_expert_axis > 1:
            if cfg.mesh_expert_axis != world:
                raise ValueError("expert parallelism spans all ranks: mesh_expert_axis must equal "
                                 f"the world size ({world})")
            if self.device.type != "cuda":
                raise ValueError("expert parallelism runs on the GPU transport")
            ep = (rank, world)
        self.model = Transformer(cfg, seed=cfg.seed if seed is None else seed, ep=ep)
        if ep is not None:
            for m in self.model.moe_layers():
                m.ep_dist = dist_ctx
                m.capacity_factor = cfg.capacity_factor
        if (dist_ctx is not None and world > 1 and cfg.mesh_expert_axis <= 1
                and cfg.expert_weights == "fused_gather" and cfg.fused_comm
                and self.device.type == "cuda" and cfg.n_experts % world == 0):
            # expert weights sharded by expert; gathered inside the grouped GEMMs
            for m in self.model.moe_layers():
                for p in (m.expert_w_gate, m.expert_w_up, m.expert_w_down):
                    p._fsdp_gather = True
        if dist_ctx is not None and world > 1:
            from .parallel.fsdp import FSDPEngine
            self.engine = FSDPEngine(self.model, cfg, self.device, dist_ctx)
        else:
            self.engine = Engine(self.model, cfg, self.device, world=1, rank=0)
        self.last_metrics = {}
        # device status word (bounded waits that ran out, bounds checks):
        # checked every step, raised as KernelStatusError one step later
        self._status = None
        if self.device.type == "cuda":
            from .ops._ext import StatusMonitor
            self._status = StatusMonitor()

    # ------------------------------------------------------------------
    def _micro_batches(self, tokens: torch.Tensor):
        B = tokens.shape[0]
        mb = self.cfg.micro_batch if self.cfg.micro_batch and self.cfg.micro_batch < B else B
        if B % mb:
            raise ValueError(f"batch {B} not divisible by micro_batch {mb}")
        return [tokens[i:i + mb] for i in range(0, B, mb)]

    def forward_backward(self, tokens: torch.Tensor):
        """Accumulate gradients of the mean loss over ``tokens`` into the flat
        gradient buffers; returns (loss, metrics) as device tensors."""
        mbs = self._micro_batches(tokens)
        n = len(mbs)
        tot = None
        metrics_acc = None
        eng = self.engine
        for i, mb in enumerate(mbs):
            if hasattr(eng, "before_forward"):
                eng.before_forward(i, n)
            with rng(f"micro{i}/forward"):
                loss, metrics = self.model.loss(mb)
            with rng(f"micro{i}/backward"):
                (loss / n).backward()
            if hasattr(eng, "after_backward"):
                eng.after_backward(i, n)
            tot = loss.detach() / n if tot is None else tot + loss.detach() / n
            if metrics_acc is None:
                metrics_acc = {k: (v / n if k != "expert_counts" else v.clone())
                               for k, v in metrics.items()}
            else:
                for k, v in metrics.items():
                    metrics_acc[k] = metrics_acc[k] + (v if k == "expert_counts" else v / n)
        return tot, metrics_acc

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """One optimizer step on ``tokens`` ``[B_local, S]``; returns the loss."""
        tokens = tokens.to(self.device, non_blocking=True).long()
        eng = self.engine
        eng.zero_grad()
        loss, metrics = self.forward_backward(tokens)
        counts = metrics["expert_counts"]
        eng.finish_step_reduce = getattr(eng, "reduce_grads", None)
        with rng("optimizer"):
            if eng.finish_step_reduce is not None:
                loss, counts = eng.reduce_grads(loss, counts)
            sq = eng.grad_sq_sum()
            if hasattr(eng, "allreduce_scalar"):
                sq = eng.allreduce_scalar(sq)
            from .optimizer import clip_coef
            coef = clip_coef(sq, self.cfg.grad_clip)
            lr = eng.apply_update(coef)
            eng.update_router_bias(counts)
        metrics["expert_counts"] = counts
        metrics["grad_norm"] = torch.sqrt(sq)
        metrics["lr"] = lr
        self.last_metrics = metrics
        if self._status is not None:
            self._status.poll()
        return loss

    def check_device_status(self):
        """Wait for the last step and raise KernelStatusError if any kernel of
        it (or before it) recorded an error."""
        if self._status is not None:
            self._status.poll()
            self._status.flush()

    # ------------------------------------------------------------------
    def state_dict(self):
        return {"params": self.engine.master_state(),
                "optimizer": self.engine.optimizer_state(),
                "step": self.engine.step_count}

    def load_state_dict(self, st):
        self.engine.load_master_state(st["params"])
        self.engine.load_optimizer_state(st["optimizer"])
        self.engine.step_count = int(st["step"])


def train(config: Config, use_random_data: bool = True, save: bool = True, dist_ctx=None,
          resume: bool = False, log=print):
    """Training loop with the reference's log line (train.py:423-562)."""
    from .checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
    from .data import SyntheticLoader
    rank = dist_ctx.rank if dist_ctx else 0
    world = dist_ctx.world if dist_ctx else 1
    is_main = rank == 0
    log = log if is_main else (lambda *a, **k: None)
    t_init = time.time()
    trainer = Trainer(config, dist_ctx=dist_ctx)
    log(f"[train] config={config.name} device={trainer.device} world={world}")
    log(f"[train] Layer attention types: {config.layer_types()}")
    log(f"[train] Trainable params: {fl.count_model_params(trainer.model):,}")
    start_step = 0
    loader = SyntheticLoader(config.vocab_size, config.batch_size // world, config.seq_len,
                             seed=42, rank=rank, pin=trainer.device.type == "cuda")
    if resume:
        path = latest_checkpoint(config)
        if path:
            extra = load_checkpoint(trainer, path, dist_ctx)
            start_step = trainer.engine.step_count
            if "loader" in extra:
                loader.load_state_dict(extra["loader"])
            log(f"[train] resumed from {path} at step {start_step}")
    model_fl, hw_fl = fl.step_flops(config)
    peak = fl.peak_flops_per_device() * world if trainer.device.type == "cuda" else 0.0
    log(f"[train] {model_fl/1e12:.2f} TFLOP/step model, {hw_fl/1e12:.2f} with remat")
    wd = None
    if dist_ctx is not None and world > 1:
        import torch.distributed as dist
        from .parallel.watchdog import Watchdog
        wd = Watchdog(dist.distributed_c10d._get_default_store(), rank, world)
    losses = []
    it = iter(loader)
    ev0 = ev1 = None
    steps_win = 0
    t_win = time.time()
    for step in range(start_step, config.train_steps):
        if wd is not None:       # between steps: nothing of ours is in flight
            wd.tick(step)
            wd.check()
        batch = next(it)
        if trainer.device.type == "cuda" and ev0 is None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        loss = trainer.step(batch)
        steps_win += 1
        if step == start_step:
            losses.append(float(loss))
            log(f"[train] compile-free first step done in {time.time()-t_init:.1f}s "
                f"(loss {losses[-1]:.4f})")
            if trainer.device.type == "cuda":
                log(hbm_report(trainer.device))
            if trainer.device.type == "cuda":
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            t_win, steps_win = time.time(), 0
            continue
        last = step == config.train_steps - 1
        if step % config.log_every == 0 or last:
            if trainer.device.type == "cuda":
                ev1 = torch.cuda.Event(enable_timing=True)
                ev1.record()
                ev1.synchronize()
                dt = ev0.elapsed_time(ev1) / 1e3
            else:
                dt = time.time() - t_win
            if dist_ctx is not None and world > 1:
                dt = dist_ctx.max_scalar(dt)
            sec = dt / max(1, steps_win)
            tps = config.batch_size * config.seq_len / sec
            m = trainer.last_metrics
            lv = float(loss)
            losses.append(lv)
            mfu = f" | MFU {100*model_fl/sec/peak:.1f}% (hw {100*hw_fl/sec/peak:.1f}%)" if peak else ""
            log(f"  step {step:5d} | loss {lv:.4f} | ce {float(m['ce']):.4f} "
                f"| z {float(m['z_loss']):.6f} | bal {float(m['bal_loss']):.6f} "
                f"| ent {float(m['mean_entropy']):.3f} "
                f"| experts {float(m['eff_experts']):.1f}/{config.n_experts} "
                f"| lr {m['lr']:.2e} | {sec*1e3:.0f} ms/step | tok/s {tps:,.0f}{mfu}")
            if config.metrics_jsonl and is_main:
                rec = {"step": step, "loss": lv, "ce": float(m["ce"]), "z_loss": float(m["z_loss"]),
                       "bal_loss": float(m["bal_loss"]), "mean_entropy": float(m["mean_entropy"]),
                       "eff_experts": float(m["eff_experts"]), "grad_norm": float(m["grad_norm"]),
                       "lr": float(m["lr"]), "ms_per_step": sec * 1e3, "tokens_per_s": tps,
                       "time": time.time()}
                if peak:
                    rec["mfu"] = model_fl / sec / peak
                    rec["hw_mfu"] = hw_fl / sec / peak
                if trainer.device.type == "cuda":
                    rec.update(hbm_stats(trainer.device))
                with open(config.metrics_jsonl, "a") as f:
                    f.write(json.dumps(rec) + "\n")
            if trainer.device.type == "cuda":
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            t_win, steps_win = time.time(), 0
        if config.checkpoint_every and (step + 1) % config.checkpoint_every == 0 and save:
            save_checkpoint(trainer, config, step + 1, dist_ctx, extra={"loader": loader.state_dict()})
        if config.gen_every and (step % config.gen_every == 0 or last) and is_main:
            from .generate import generate_from_model
            from .data import get_tokenizer
            text, _ = generate_from_model(trainer.model, config, get_tokenizer(config),
                                          config.gen_prompt, config.gen_max_tokens,
                                          config.gen_temperature, config.gen_top_k, seed=step)
            log(f"  [gen @ step {step}] {config.gen_prompt!r} -> {text!r}")
    if save:
        save_checkpoint(trainer, config, config.train_steps, dist_ctx,
                        extra={"loader": loader.state_dict()})
    if wd is not None:
        wd.close()
    if trainer.device.type == "cuda":
        trainer.check_device_status()
        log(hbm_report(trainer.device))
    if losses:
        log(f"[train] Done. First loss={losses[0]:.4f}, last loss={losses[-1]:.4f}")
    return trainer, losses


def hbm_stats(device) -> dict:
    """Device-memory figures of this process (the reference's hbm_report,
    train.py:337-346, reads the same from the accelerator's memory stats)."""
    st = torch.cuda.memory_stats(device)
    free, total = torch.cuda.mem_get_info(device)
    gb = 1e9
    return {"hbm_in_use_gb": st.get("allocated_bytes.all.current", 0) / gb,
            "hbm_peak_gb": st.get("allocated_bytes.all.peak", 0) / gb,
            "hbm_reserved_gb": st.get("reserved_bytes.all.current", 0) / gb,
            "hbm_total_gb": total / gb, "hbm_free_gb": free / gb}


def hbm_report(device) -> str:
    h = hbm_stats(device)
    return (f"[hbm] {device}: in use {h['hbm_in_use_gb']:.2f} GB, peak {h['hbm_peak_gb']:.2f} GB, "
            f"reserved {h['hbm_reserved_gb']:.2f} GB of {h['hbm_total_gb']:.1f} GB "
            f"({h['hbm_free_gb']:.1f} GB free)")


def memory_report(config: Config) -> str:
    """Per-tensor table of the parameter tree with fp32 MB and per-device MB
    under the data-parallel shard rule (train.py:349-395), built on the meta
    device so nothing is allocated."""
    from .checkpoint import param_shapes
    shapes = param_shapes(config)
    world = max(1, config.mesh_data_axis * config.mesh_expert_axis)
    rows, total, per_dev = [], 0.0, 0.0
    for name, shape in shapes.items():
        n = 1
        for s in shape:
            n *= s
        mb = n * 4 / 1e6
        small = n < (1 << 16)
        pmb = mb if small else mb / world
        rows.append((mb, pmb, name, shape, "replicated" if small else f"state shard/{world}"))
        total += mb
        per_dev += pmb
    out = [f"layout: fp32 master + optimizer state of tensors >= 65536 elements are sharded over "
           f"the {world} data ranks; the bf16 working copy and the fp32 gradient buffers are "
           f"full on every rank",
           f"{'tensor':46s} {'shape':24s} {'layout':18s} {'fp32 MB':>9s} {'master/dev':>10s}",
           "-" * 111]
    for mb, pmb, name, shape, lay in sorted(rows, reverse=True):
        out.append(f"{name[:46]:46s} {str(tuple(shape))[:24]:24s} {lay:18s} {mb:9.1f} {pmb:10.1f}")
    out.append("-" * 111)
    out.append(f"{'TOTAL':46s} {'':24s} {'':18s} {total:9.1f} {per_dev:10.1f}")
    opt_mult = 2 if config.optimizer == "adamw" else (0.5 if config.opt_state_dtype == "bf16" else 1)
    out.append(f"per device: master {per_dev/1e3:.2f} GB + optimizer {per_dev*opt_mult/1e3:.2f} GB "
               f"({config.optimizer}) + bf16 working copy {total/2/1e3:.2f} GB + fp32 grads "
               f"{total/1e3:.2f} GB")
    m, h = fl.step_flops(config)
    out.append(f"step FLOPs: {m/1e12:.1f} T model, {h/1e12:.1f} T with remat")
    return "\n".join(out)
