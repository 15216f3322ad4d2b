"""Training engine: flat parameter storage, gradient accumulation, clipping,
fused optimizer update and the router-bias balancing rule.

Storage.  Parameters are grouped into *units* (the embedding, each block, the
final norm) and, inside a unit, by compute dtype: matrices run in the compute
dtype (bf16), everything small (norm scales, conv taps, gate biases, decay
parameters, residual scales, router) in fp32.  Each group owns

    master  fp32, the local shard [lo, hi) of the padded flat vector
    work    compute dtype, full length  (what the kernels read)
    grad    fp32, full length            (what the kernels accumulate into)
    m, v    optimizer state, local shard

and every ``nn.Parameter`` of the model is re-pointed at its slice of
``work`` (``p.data``), with ``p.main_grad``/``p.grad`` at its slice of
``grad``.  With one rank the shard is the whole vector; with data parallelism
the engine in :mod:`hanuman_b200.parallel.fsdp` reduce-scatters ``grad`` into
the shard and all-gathers the updated ``work``.

The step follows train.py:220-323: loss over micro-batches, clip by global
norm, Lion/AdamW with lr-scaled decoupled weight decay, then
``bias -= rate * sign(count - mean(count))`` per MoE layer.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn

from . import optimizer as optim
from .config import Config

ALIGN = 64  # elements; keeps every parameter slice 128-byte aligned in bf16


def _is_matrix(name: str, p: torch.Tensor) -> bool:
    """Parameters computed in the compute dtype by GEMM kernels."""
    if p.dim() < 2:
        return False
    leaf = name.split(".")[-1]
    if leaf in ("router", "weight"):  # router GEMM and conv taps stay fp32
        return False
    if leaf in ("f_proj0", "f_proj1", "g_proj0", "g_proj1", "wb"):
        return True
    return True


@dataclass
class FlatGroup:
    names: list
    params: list
    offsets: list
    numel: int           # padded total
    dtype: torch.dtype   # work dtype
    work: torch.Tensor = None
    grad: torch.Tensor = None
    master: torch.Tensor = None
    m: torch.Tensor = None
    v: torch.Tensor = None
    decay: torch.Tensor = None
    lo: int = 0
    hi: int = 0
    trainable: torch.Tensor = None  # 1.0 where the element receives updates
    local: bool = False             # expert-parallel slice owned by this rank only
    gathered: bool = False          # one expert-weight tensor, shards = whole experts,
                                    # gathered by the consuming grouped GEMM
    matrices: bool = False          # the unit's GEMM-weight group
    sharded: bool = False           # FSDP: only `shard` persists; `work` is gathered for use
    shard: torch.Tensor = None      # this rank's slice [lo, hi) of the working copy


def _build_group(named, dtype, device, world, rank, master_init) -> Optional[FlatGroup]:
    if not named:
        return None
    offsets, off = [], 0
    for _, p in named:
        offsets.append(off)
        off += (p.numel() + ALIGN - 1) // ALIGN * ALIGN
    per = ALIGN * world
    numel = (off + per - 1) // per * per
    g = FlatGroup([n for n, _ in named], [p for _, p in named], offsets, numel, dtype)
    shard = numel // world
    g.lo, g.hi = rank * shard, (rank + 1) * shard
    full_master = torch.zeros(numel, dtype=torch.float32)
    decay = torch.zeros(numel, dtype=torch.float32)
    trainable = torch.zeros(numel, dtype=torch.float32)
    for (n, p), o in zip(named, offsets):
        full_master[o:o + p.numel()] = master_init[n].reshape(-1)
        if not optim.is_no_decay(n):
            decay[o:o + p.numel()] = 1.0
        if p.requires_grad:
            trainable[o:o + p.numel()] = 1.0
    g.master = full_master[g.lo:g.hi].clone().to(device)
    g.decay = decay[g.lo:g.hi].clone().to(device)
    g.trainable = trainable[g.lo:g.hi].clone().to(device)
    g.work = full_master.to(device=device, dtype=dtype)
    g.grad = torch.zeros(numel, dtype=torch.float32, device=device)
    for (n, p), o in zip(named, offsets):
        p.data = g.work[o:o + p.numel()].view(p.shape)
        gv = g.grad[o:o + p.numel()].view(p.shape)
        p.main_grad = gv
        if p.requires_grad:
            p.grad = gv if dtype == torch.float32 else None
    return g


class Engine:
    """Owns the flat buffers and the optimizer for one rank."""

    def __init__(self, model: nn.Module, cfg: Config, device: torch.device,
                 world: int = 1, rank: int = 0):
        self.model = model
        self.cfg = cfg
        self.device = torch.device(device)
        self.world, self.rank = world, rank
        self.step_count = 0
        self.schedule = optim.schedule_for(cfg)
        cdt = cfg.compute_dtype()
        if self.device.type == "cpu":
            # CPU path: fp32 parameters cast at use, like the reference
            cdt = torch.float32
        master_init = {n: p.detach().float().clone() for n, p in model.named_parameters()}
        model.to(self.device)
        self.units = self._units(model)
        self.groups: list[FlatGroup] = []
        self.unit_groups: list[list[int]] = []   # group indices of each unit
        for unit in self.units:
            first = len(self.groups)
            local = [(n, p) for n, p in unit if getattr(p, "_ep_local", False)]
            rest = [(n, p) for n, p in unit if not getattr(p, "_ep_local", False)]
            gath = [(n, p) for n, p in rest if getattr(p, "_fsdp_gather", False)]
            rest = [(n, p) for n, p in rest if not getattr(p, "_fsdp_gather", False)]
            for n, p in gath:   # one group per tensor: the shards are whole experts
                g = _build_group([(n, p)], cdt, self.device, world, rank, master_init)
                g.gathered = g.numel == p.numel() and p.shape[0] % world == 0
                self.groups.append(g)
            mats = [(n, p) for n, p in rest if _is_matrix(n, p)]
            smalls = [(n, p) for n, p in rest if not _is_matrix(n, p)]
            for named, dt, loc in ((mats, cdt, False), (smalls, torch.float32, False),
                                   (local, cdt, True)):
                g = _build_group(named, dt, self.device, 1 if loc else world, 0 if loc else rank,
                                 master_init)
                if g is not None:
                    g.local = loc
                    g.matrices = named is mats
                    self.groups.append(g)
            self.unit_groups.append(list(range(first, len(self.groups))))
        mdt = torch.bfloat16 if (cfg.optimizer == "lion" and cfg.opt_state_dtype == "bf16") \
            else torch.float32
        for g in self.groups:
            g.m = torch.zeros(g.hi - g.lo, dtype=mdt, device=self.device)
            if cfg.optimizer == "adamw":
                g.v = torch.zeros(g.hi - g.lo, dtype=torch.float32, device=self.device)
        self.param_index = {}
        for gi, g in enumerate(self.groups):
            for n, o, p in zip(g.names, g.offsets, g.params):
                self.param_index[n] = (gi, o, p.numel(), tuple(p.shape))
        self._bias_params = [(i, m.bias) for i, m in enumerate(model.moe_layers())]

    # ------------------------------------------------------------------
    @staticmethod
    def _units(model):
        """[(name, param)] lists: wte, each block, then the rest."""
        named = list(model.named_parameters())
        units, used = [], set()
        units.append([(n, p) for n, p in named if n == "wte"])
        used.add("wte")
        for i in range(len(model.blocks)):
            pre = f"blocks.{i}."
            u = [(n, p) for n, p in named if n.startswith(pre)]
            units.append(u)
            used.update(n for n, _ in u)
        rest = [(n, p) for n, p in named if n not in used]
        if rest:
            units.append(rest)
        return [u for u in units if u]

    def zero_grad(self):
        for g in self.groups:
            g.grad.zero_()

    # ------------------------------------------------------------------
    def grad_sq_sum(self) -> torch.Tensor:
        """Sum of squared (already reduced) gradients over this rank's shards."""
        if self.device.type == "cuda":
            from .ops.optim import sumsq_cuda
            return sumsq_cuda([g.grad[g.lo:g.hi] for g in self.groups])
        tot = torch.zeros((), dtype=torch.float64, device=self.device)
        for g in self.groups:
            tot += g.grad[g.lo:g.hi].double().pow(2).sum()
        return tot.float()

    def apply_update(self, coef: torch.Tensor):
        """Optimizer update on the shards, then refresh the working copy."""
        cfg = self.cfg
        lr = self.schedule(self.step_count)
        self.step_count += 1
        if self.device.type == "cuda":
            from .ops.optim import fused_update_cuda
            for g in self.groups:
                fused_update_cuda(g, cfg, lr, self.step_count, coef)
            return lr
        for g in self.groups:
            gs = g.grad[g.lo:g.hi]
            if cfg.optimizer == "lion":
                optim.lion_update_(g.master, gs, g.m, g.decay, lr, cfg.weight_decay,
                                   cfg.lion_b1, cfg.lion_b2, coef)
            else:
                optim.adamw_update_(g.master, gs, g.m, g.v, g.decay, lr, cfg.weight_decay,
                                    cfg.adam_b1, cfg.adam_b2, cfg.adam_eps, self.step_count,
                                    coef)
            (g.shard if g.sharded else g.work[g.lo:g.hi]).copy_(g.master.to(g.work.dtype))
        return lr

    @torch.no_grad()
    def update_router_bias(self, counts: torch.Tensor):
        """bias -= rate * sign(count - layer mean), per MoE layer (train.py:242-260)."""
        if not self._bias_params or counts.numel() == 0:
            return
        delta = self.cfg.bias_update_rate * torch.sign(counts - counts.mean(-1, keepdim=True))
        for i, b in self._bias_params:
            gi, o, n, _ = self.param_index[self._bias_name(i)]
            g = self.groups[gi]
            b.data.sub_(delta[i].to(b.dtype))   # working copy (full, fp32)
            lo, hi = max(o, g.lo), min(o + n, g.hi)
            if lo < hi:                         # master element range owned here
                g.master[lo - g.lo:hi - g.lo].sub_(delta[i][lo - o:hi - o].float())

    def _bias_name(self, i):
        if not hasattr(self, "_bias_names"):
            self._bias_names = [n for n, _ in self.model.named_parameters()
                                if n.endswith("ffn.bias")]
        return self._bias_names[i]

    # ------------------------------------------------------------------
    def master_state(self) -> dict:
        """Full fp32 master weights by reference-tree name (gathers shards; the
        expert-parallel slices are concatenated along the expert axis)."""
        out = {}
        for g in self.groups:
            full = self._gather_master(g)
            for n, o, p in zip(g.names, g.offsets, g.params):
                if g.local and self.world > 1:
                    parts = [full[r][o:o + p.numel()].view(p.shape) for r in range(self.world)]
                    out[n] = torch.cat(parts, 0).clone()
                else:
                    out[n] = full[o:o + p.numel()].view(p.shape).clone()
        return out

    def _gather_master(self, g: FlatGroup):
        if g.local and self.world > 1:
            import torch.distributed as dist
            parts = [torch.empty_like(g.master) for _ in range(self.world)]
            dist.all_gather(parts, g.master)
            return parts
        if self.world == 1 or g.local:
            return g.master
        import torch.distributed as dist
        full = torch.empty(g.numel, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, g.master)
        return full

    def load_master_state(self, state: dict):
        for g in self.groups:
            full = torch.zeros(g.numel, dtype=torch.float32, device=self.device)
            for n, o, p in zip(g.names, g.offsets, g.params):
                v = state[n]
                if g.local and tuple(v.shape) != tuple(p.shape):  # full tensor -> own experts
                    nl = p.shape[0]
                    v = v[self.rank * nl:(self.rank + 1) * nl]
                full[o:o + p.numel()] = v.reshape(-1).to(self.device, torch.float32)
            g.master.copy_(full[g.lo:g.hi])
            if g.sharded:
                g.shard.copy_(full[g.lo:g.hi].to(g.shard.dtype))
            else:
                g.work.copy_(full.to(g.work.dtype))

    def optimizer_state(self) -> dict:
        return {f"group{i}": {"m": g.m, **({"v": g.v} if g.v is not None else {})}
                for i, g in enumerate(self.groups)}

    def load_optimizer_state(self, st: dict):
        for i, g in enumerate(self.groups):
            d = st[f"group{i}"]
            g.m.copy_(d["m"])
            if g.v is not None:
                g.v.copy_(d["v"])
