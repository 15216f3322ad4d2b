"""Data-parallel training engine with sharded master weights and optimizer state.

Layout (per flat group, see :mod:`hanuman_b200.engine`): every rank owns the
fp32 master and the optimizer moments of ONE contiguous 1/world slice
``[lo, hi)`` of the padded flat vector, and holds the full compute-dtype
working copy and the full fp32 gradient buffer.  The reference's FSDP
(model/sharding.py:67-113: shard the parameters, gather them for use,
reduce-scatter the gradients) maps to:

    backward         gradients accumulate locally into the full grad buffer
    reduce_grads     grad[lo:hi] <- mean over ranks   (reduce-scatter)
    grad_sq_sum      sum of squares of the local shard, all-reduced (clip norm)
    apply_update     Lion/AdamW on the shard -> new master[lo:hi], work[lo:hi]
    gather_work      work <- concatenation of every rank's work[lo:hi] (all-gather)

Two transports implement the two collectives:

* ``nccl`` (baseline): ``reduce_scatter_tensor`` / ``all_gather_into_tensor``.
* ``p2p`` (fused): the gradient buffers live in symmetric memory; one kernel
  reads every peer's slice of the gradient over NVLink, sums it, scales it and
  emits the shard's sum of squares; the update kernel writes the new bf16
  working values into EVERY peer's working copy with peer stores, so the
  all-gather disappears into the optimizer.  Selected with ``cfg.fused_comm``
  when symmetric memory is available; otherwise NCCL.
* ``expert_weights = "fused_gather"`` (with ``p2p``): the MoE expert tensors
  are sharded by expert and only their owner updates them; the forward's
  grouped GEMMs pull the other experts' tiles from the owners' memory
  (model/moe.py:202-245 gathers them with ``all_gather(tiled)`` instead).

With 180 GB per GPU the full working copy stays resident (no re-gather in the
backward), which is what makes the all-gather a once-per-step operation.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import Config
from ..engine import Engine


class FSDPEngine(Engine):
    def __init__(self, model, cfg: Config, device, ctx):
        self.ctx = ctx
        super().__init__(model, cfg, device, world=ctx.world, rank=ctx.rank)
        self.transport = "nccl"
        self.p2p = None
        if cfg.fused_comm and self.device.type == "cuda":
            try:
                from .p2p import P2PComm
                self.p2p = P2PComm(self, ctx)
                self.transport = "p2p"
            except Exception as e:  # pragma: no cover - depends on the box
                if ctx.rank == 0:
                    print(f"[fsdp] fused peer-memory transport unavailable ({e}); using NCCL")
                self.p2p = None
        self._attach_expert_gather()

    def _attach_expert_gather(self):
        """Hand each MoE layer the shard addresses of its gathered expert tensors."""
        gathered = [g for g in self.groups if g.gathered]
        if not gathered:
            return
        if self.p2p is None:
            # no peer memory: these groups fall back to the NCCL all-gather
            for g in gathered:
                g.gathered = False
            return
        from ..ops.moe import ExpertGather
        by_layer = {}
        for g in gathered:
            name = g.names[0]
            layer, leaf = name.rsplit(".", 1)
            by_layer.setdefault(layer, {})[leaf] = (self.p2p.gather_ptrs[name], g.params[0])
        for layer, d in by_layer.items():
            mod = self.model.get_submodule(layer)
            if set(d) != {"expert_w_gate", "expert_w_up", "expert_w_down"}:
                raise RuntimeError(f"{layer}: expert tensors must all be gathered")
            N = d["expert_w_gate"][1].shape[0]
            mod._gather = ExpertGather({k: v[0] for k, v in d.items()}, self.rank, N // self.world,
                                       {k: tuple(v[1].shape) for k, v in d.items()}, self.device)

    # ------------------------------------------------------------------
    def reduce_grads(self, loss, counts):
        """Mean gradient over ranks into each group's shard; global counts/loss."""
        w = self.world
        for g in self.groups:
            if g.local:  # expert-parallel slice: the owner saw every token; mean over ranks
                g.grad.mul_(1.0 / w)
        if self.p2p is not None:
            self.p2p.reduce_scatter_grads()
        else:
            for g in self.groups:
                if g.local:
                    continue
                shard = g.grad[g.lo:g.hi]
                if self.ctx.backend == "nccl":
                    dist.reduce_scatter_tensor(shard, g.grad, op=dist.ReduceOp.SUM)
                else:  # gloo (CPU ranks): all-reduce, keep the owned slice
                    dist.all_reduce(g.grad, op=dist.ReduceOp.SUM)
                shard.mul_(1.0 / w)
        packed = torch.cat([loss.detach().reshape(1).float(), counts.reshape(-1).float()])
        dist.all_reduce(packed, op=dist.ReduceOp.SUM)
        loss = packed[0] / w
        counts = packed[1:].view_as(counts)
        return loss, counts

    def grad_sq_sum(self):
        if self.p2p is not None and self.p2p.sumsq is not None:
            tot = self.p2p.sumsq.reshape(())
            loc = [g.grad for g in self.groups if g.local]
            if loc:
                from ..ops.optim import sumsq_cuda
                tot = tot + sumsq_cuda(loc)
            return tot
        return super().grad_sq_sum()

    def allreduce_scalar(self, x):
        t = x.reshape(1).float().clone()
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.reshape(())

    def apply_update(self, coef):
        if self.p2p is not None:
            lr = self.schedule(self.step_count)
            self.step_count += 1
            self.p2p.update_and_broadcast(self.cfg, lr, self.step_count, coef)
            from ..ops.optim import fused_update_cuda
            for g in self.groups:
                if g.local:
                    fused_update_cuda(g, self.cfg, lr, self.step_count, coef)
            return lr
        lr = super().apply_update(coef)
        self.gather_work()
        return lr

    def gather_work(self):
        for g in self.groups:
            if g.local:
                continue
            dist.all_gather_into_tensor(g.work, g.work[g.lo:g.hi].clone()
                                        if self.device.type == "cpu" else g.work[g.lo:g.hi])

    def update_router_bias(self, counts):
        # counts are already summed over ranks: every rank applies the same delta
        # to its full working copy and to the part of the master it owns.
        super().update_router_bias(counts)
