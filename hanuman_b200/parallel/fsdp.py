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

FSDP (``cfg.shard_params``, the default with more than one rank): the
compute-dtype working copy of each unit's matrices is sharded too.  Only the
rank's slice (``shard``, in symmetric memory on the fused transport) persists;
the model calls ``pre_forward`` / ``post_forward`` around each block and the
block-boundary autograd nodes call ``pre_backward`` / ``post_backward``, and the
engine gathers the unit's full weights into the storage of its ``work`` tensor
before each use (on the fused transport, one copy-engine ``cudaMemcpyAsync``
per rank from every rank's shard in symmetric memory, so a prefetch of the
next unit on a side stream takes no SM time from the unit that computes; or
NCCL ``all_gather_into_tensor``) and releases that storage afterwards.  The
parameters and the weight views saved for the backward keep pointing at the
same storage object, which is re-filled before the unit's backward.  The
optimizer writes only the local shard; the embedding stays gathered from the
first forward to the end of the backward (the tied head reads it).

Overlap (``cfg.overlap_reduce``): during the last micro-batch's backward the
model calls ``post_backward(unit)`` as soon as a block's gradients are final
(an identity autograd node at the block's input, models/transformer.py), and
that block's reduce-scatter starts while the backward of the earlier blocks
runs: NCCL ``reduce_scatter_tensor(async_op=True)``, or on the fused transport
a comm stream that waits for the block's gradients, runs the device barrier and
the peer-reading reduce-scatter kernel.  ``reduce_grads`` reduces the units not
reduced yet (the embedding, whose last gradient is the embedding backward, and
the final norm) and joins the outstanding work.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import Config
from ..engine import Engine


def ext_copy_gather(addrs, shard_bytes, out):
    from ..ops._ext import ext
    ext().copy_engine_gather(list(addrs), shard_bytes, out)


class FSDPEngine(Engine):
    def __init__(self, model, cfg: Config, device, ctx):
        self.ctx = ctx
        super().__init__(model, cfg, device, world=ctx.world, rank=ctx.rank)
        self._gathered_units: set[int] = set()
        self._prefetch_ev: dict[int, object] = {}
        self._pf_stream = None
        self._shard_units()
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
        self._last_micro = False
        self._reduced: set[int] = set()
        self._pending = []          # NCCL work handles of this step
        self._comm_stream = None
        if cfg.overlap_reduce or self.sharded_units:
            model.unit_hooks = self
        if cfg.overlap_reduce and self.p2p is not None:
            self._comm_stream = torch.cuda.Stream(device=self.device)

    # ------------------------------------------------------------------
    # FSDP: sharded working weights
    def _shard_units(self):
        """Keep only this rank's slice of every unit's matrix group; the full
        ``work`` tensor (which the parameters view) gets its storage only while
        the unit is in use."""
        self.sharded_units: dict[int, list] = {}
        if not self.cfg.shard_params or self.world <= 1:
            return
        for u, idx in enumerate(self.unit_groups):
            for i in idx:
                g = self.groups[i]
                if g.local or g.gathered or not g.matrices:
                    continue
                g.sharded = True
                g.shard = g.work[g.lo:g.hi].clone()
                g.full_bytes = g.numel * g.work.element_size()
                g.work.untyped_storage().resize_(0)
                self.sharded_units.setdefault(u, []).append(g)

    def gather_unit(self, unit: int):
        """Full working weights of ``unit`` from every rank's shard (no-op if
        the unit holds none or is gathered already; a prefetched unit makes the
        current stream wait for its gather)."""
        groups = self.sharded_units.get(unit)
        if not groups:
            return
        if unit in self._gathered_units:
            ev = self._prefetch_ev.pop(unit, None)
            if ev is not None:
                torch.cuda.current_stream().wait_event(ev)
            return
        self._gathered_units.add(unit)
        self._fill(groups)

    def prefetch_unit(self, unit: int):
        """Start gathering ``unit`` on the prefetch stream, behind everything the
        compute stream has enqueued so far, so that it overlaps the compute of
        the unit in progress."""
        groups = self.sharded_units.get(unit)
        if not groups or unit in self._gathered_units or self.device.type != "cuda":
            return
        self._gathered_units.add(unit)
        main = torch.cuda.current_stream()
        if self._pf_stream is None:
            self._pf_stream = torch.cuda.Stream(device=self.device)
        self._pf_stream.wait_stream(main)
        with torch.cuda.stream(self._pf_stream):
            self._fill(groups, record=main)
            ev = torch.cuda.Event()
            ev.record()
        self._prefetch_ev[unit] = ev

    def _fill(self, groups, record=None):
        for g in groups:
            st = g.work.untyped_storage()
            st.resize_(g.full_bytes)
            if record is not None:   # allocated on the prefetch stream, used on `record`
                g.work.record_stream(record)
            if self.p2p is not None:
                # copy engines read every rank's shard (peer addresses of the
                # symmetric buffers): no SM time, so a prefetch overlaps compute
                ext_copy_gather(self.p2p.shard_addrs[id(g)], (g.hi - g.lo) * g.work.element_size(), g.work)
            else:
                # the collective bumps its output's version counter, which
                # autograd checks on the weight views saved for the backward:
                # gather into a temporary and copy at the storage level
                tmp = torch.empty(g.numel, dtype=g.work.dtype, device=g.work.device)
                dist.all_gather_into_tensor(tmp, g.shard)
                st.copy_(tmp.untyped_storage())

    def free_unit(self, unit: int):
        if unit not in self._gathered_units:
            return
        ev = self._prefetch_ev.pop(unit, None)
        if ev is not None:          # never used: still order the release after its gather
            torch.cuda.current_stream().wait_event(ev)
        self._gathered_units.discard(unit)
        for g in self.sharded_units.get(unit, ()):
            g.work.untyped_storage().resize_(0)

    def gathered_all(self):
        """Context manager: every unit's weights gathered (evaluation, sampling)."""
        import contextlib

        @contextlib.contextmanager
        def cm():
            for u in self.sharded_units:
                self.gather_unit(u)
            try:
                yield
            finally:
                for u in list(self.sharded_units):
                    self.free_unit(u)
        return cm()

    def pre_forward(self, unit: int):
        self.gather_unit(unit)
        self.prefetch_unit(unit + 1)

    def post_forward(self, unit: int):
        # the embedding stays gathered through the tied head (freed after the
        # backward); a block is re-gathered for its backward
        if unit != 0:
            self.free_unit(unit)

    # ------------------------------------------------------------------
    # unit hooks (called from the model's backward)
    def before_forward(self, i, n):
        self._last_micro = i == n - 1

    def pre_backward(self, unit: int):
        self.gather_unit(unit)
        if unit > 1:
            self.prefetch_unit(unit - 1)

    def post_backward(self, unit: int):
        """All gradients of ``unit`` are final for this micro-batch; free its
        gathered weights and, on the last one, start its reduce-scatter."""
        self.free_unit(unit)
        if self.cfg.overlap_reduce and self._last_micro and unit not in self._reduced:
            self._reduce_unit(unit)

    def _reduce_unit(self, unit: int):
        first = not self._reduced
        self._reduced.add(unit)
        if first and self.p2p is not None:
            self.p2p.begin_step()   # zeroed sum of squares, on the compute stream
        groups = [self.groups[i] for i in self.unit_groups[unit] if not self.groups[i].local]
        if not groups:
            return
        if self.p2p is not None:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self._comm_stream or torch.cuda.current_stream()):
                if self._comm_stream is not None:
                    self._comm_stream.wait_event(ev)
                self.p2p.reduce_scatter_groups(groups)
            return
        for g in groups:
            shard = g.grad[g.lo:g.hi]
            if self.ctx.backend == "nccl":
                h = dist.reduce_scatter_tensor(shard, g.grad, op=dist.ReduceOp.SUM, async_op=True)
            else:  # gloo (CPU ranks): all-reduce, keep the owned slice
                h = dist.all_reduce(g.grad, op=dist.ReduceOp.SUM, async_op=True)
            self._pending.append((h, g))

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
        for u in list(self._gathered_units):   # the embedding (kept for the tied head)
            self.free_unit(u)
        for g in self.groups:
            if g.local:  # expert-parallel slice: the owner saw every token; mean over ranks
                g.grad.mul_(1.0 / w)
        if self.cfg.overlap_reduce:
            for u in range(len(self.unit_groups)):   # units the backward did not reduce
                if u not in self._reduced:
                    self._reduce_unit(u)
            if self.p2p is not None:
                with torch.cuda.stream(self._comm_stream or torch.cuda.current_stream()):
                    self.p2p.end_reduce()
                if self._comm_stream is not None:
                    torch.cuda.current_stream().wait_stream(self._comm_stream)
            for h, g in self._pending:
                h.wait()
                g.grad[g.lo:g.hi].mul_(1.0 / w)
            self._pending = []
            self._reduced = set()
        elif self.p2p is not None:
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
            if g.local or g.sharded:   # sharded units are gathered at their next use
                continue
            dist.all_gather_into_tensor(g.work, g.work[g.lo:g.hi].clone()
                                        if self.device.type == "cpu" else g.work[g.lo:g.hi])

    def update_router_bias(self, counts):
        # counts are already summed over ranks: every rank applies the same delta
        # to its full working copy and to the part of the master it owns.
        super().update_router_bias(counts)
