"""Symmetric-memory transport for the data-parallel engine.

All gradient buffers (fp32) and working-weight buffers (bf16 / fp32) of an
engine are re-homed into three symmetric-memory allocations, so every rank knows
the device address of every peer's copy.  The step then runs three native
kernels per flat group and three device-side barriers per step:

    barrier -> p2p_reduce_scatter (peer loads, sum, scale, sum of squares)
            -> barrier -> ... optimizer: p2p_update_bcast (peer stores of the
               new working values into every rank's copy) -> barrier

No host synchronisation and no NCCL call is on this path except the one-float
all-reduce of the squared gradient norm.

Expert-weight tensors marked for the fused gather (``expert_weights =
"fused_gather"``) are updated in place on their owner only; their forward
consumers pull the other ranks' experts over NVLink inside the grouped GEMM
(``grouped_gemm_m_gather``), so for them the all-gather moves from the
optimizer into the first GEMM that needs the weights.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext


class P2PComm:
    def __init__(self, eng, ctx):
        import torch.distributed._symmetric_memory as symm
        self.eng, self.ctx = eng, ctx
        self.world, self.rank = ctx.world, ctx.rank
        dev = eng.device
        group = dist.group.WORLD
        groups = [g for g in eng.groups if not g.local]
        self.groups = groups
        # one symmetric allocation per buffer kind
        gtot = sum(g.numel for g in groups)
        self.gbuf = symm.empty(gtot, dtype=torch.float32, device=dev)
        self.gbuf.zero_()
        self.ghdl = symm.rendezvous(self.gbuf, group)
        kinds = {}
        for g in groups:
            kinds.setdefault(g.work.dtype, 0)
            kinds[g.work.dtype] += (g.hi - g.lo) if g.sharded else g.numel
        self.wbuf, self.whdl = {}, {}
        for dt, n in kinds.items():
            t = symm.empty(n, dtype=dt, device=dev)
            self.wbuf[dt] = t
            self.whdl[dt] = symm.rendezvous(t, group)
        self.flags = symm.empty(max(self.world, 32), dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.fhdl = symm.rendezvous(self.flags, group)
        torch.cuda.synchronize(dev)
        dist.barrier()
        # re-home every group and re-point the parameters
        goff, woff = 0, {dt: 0 for dt in kinds}
        self.layout = []
        self.gather_ptrs = {}   # gathered tensor name -> every rank's shard address
        self.shard_ptrs = {}    # id(sharded group) -> every rank's shard address (device tensor)
        self.shard_addrs = {}   # the same addresses as host integers (copy-engine gather)
        for g in groups:
            dt = g.work.dtype
            nw = (g.hi - g.lo) if g.sharded else g.numel
            new_grad = self.gbuf[goff:goff + g.numel]
            new_work = self.wbuf[dt][woff[dt]:woff[dt] + nw]
            new_grad.copy_(g.grad)
            g.grad = new_grad
            if g.sharded:   # FSDP: the shard is symmetric; the full buffer stays local
                new_work.copy_(g.shard)
                g.shard = new_work
            else:
                new_work.copy_(g.work)
                g.work = new_work
            for n, o, p in zip(g.names, g.offsets, g.params):
                if not g.sharded:
                    p.data = g.work[o:o + p.numel()].view(p.shape)
                gv = g.grad[o:o + p.numel()].view(p.shape)
                p.main_grad = gv
                if p.requires_grad and dt == torch.float32:
                    p.grad = gv
            esz_w = torch.tensor([], dtype=dt).element_size()
            gp = torch.tensor([int(self.ghdl.buffer_ptrs[r]) + goff * 4 for r in range(self.world)],
                              dtype=torch.int64, device=dev)
            bases = [int(self.whdl[dt].buffer_ptrs[r]) + woff[dt] * esz_w for r in range(self.world)]
            if g.sharded:
                # the update writes this rank's shard (its element lo + i sits at
                # shard + i); peers read the shards to gather the unit
                wp = torch.tensor([bases[self.rank] - g.lo * esz_w], dtype=torch.int64, device=dev)
                self.shard_ptrs[id(g)] = torch.tensor(bases, dtype=torch.int64, device=dev)
                self.shard_addrs[id(g)] = bases
            elif g.gathered:
                # the update stays local; peers pull this shard in their forward
                wp = torch.tensor([bases[self.rank]], dtype=torch.int64, device=dev)
                shard = g.numel // self.world
                self.gather_ptrs[g.names[0]] = [bases[r] + r * shard * esz_w for r in range(self.world)]
            else:
                wp = torch.tensor(bases, dtype=torch.int64, device=dev)
            self.layout.append((gp, wp))
            goff += g.numel
            woff[dt] += nw
        self.pads = torch.tensor([int(p) for p in self.fhdl.buffer_ptrs], dtype=torch.int64, device=dev)
        self.epoch = 0
        self.sumsq = None
        torch.cuda.synchronize(dev)
        dist.barrier()

    def barrier(self):
        self.epoch += 1
        ext().p2p_barrier(self.pads, self.rank, self.world, self.epoch)

    def reduce_scatter_grads(self):
        self.barrier()                      # every rank's backward is complete
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=self.eng.device)
        for g, (gp, _) in zip(self.groups, self.layout):
            ext().p2p_reduce_scatter(gp, self.world, g.lo, g.hi - g.lo, g.grad[g.lo:g.hi],
                                     1.0 / self.world, self.sumsq)
        self.barrier()                      # nobody reads a peer's gradients any more

    # per-unit reduce-scatter (overlapped with the backward, on the caller's stream)
    def begin_step(self):
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=self.eng.device)

    def reduce_scatter_groups(self, groups):
        """Barrier (every rank's gradients of these groups are final), then the
        peer-reading reduce-scatter of each group into its shard."""
        self.barrier()
        index = {id(g): i for i, g in enumerate(self.groups)}
        for g in groups:
            gp, _ = self.layout[index[id(g)]]
            ext().p2p_reduce_scatter(gp, self.world, g.lo, g.hi - g.lo, g.grad[g.lo:g.hi],
                                     1.0 / self.world, self.sumsq)

    def end_reduce(self):
        self.barrier()                      # nobody reads a peer's gradients any more

    def update_and_broadcast(self, cfg, lr, step, coef):
        mode = 0 if cfg.optimizer == "adamw" else 1
        b1 = cfg.adam_b1 if mode == 0 else cfg.lion_b1
        b2 = cfg.adam_b2 if mode == 0 else cfg.lion_b2
        c = coef.reshape(1).float().contiguous()
        for g, (_, wp) in zip(self.groups, self.layout):
            ext().p2p_update_bcast(g.master, g.grad[g.lo:g.hi], g.m, g.v, g.decay, wp,
                                   1 if (g.gathered or g.sharded) else self.world,
                                   g.lo, g.work.dtype == torch.bfloat16, mode, float(lr),
                                   float(cfg.weight_decay), float(b1), float(b2),
                                   float(cfg.adam_eps), int(step), c)
        self.barrier()                      # every rank's copy is fully written
